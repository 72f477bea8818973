/*
 * mogemma_b200.h -- C ABI of libmogemma_cuda.so, the B200 (sm_100a) Gemma 3
 * forward/decode engine that replaces the MoGemma Mojo engine behind the
 * `mogemma._core` operator boundary.
 *
 * Conventions
 *   - Every entry point returns mg_status; on failure mg_last_error() returns a
 *     thread-local message.  Messages that the reference raises keep its wording
 *     ("Sequence length exceeded", core.mojo:380-381).
 *   - Pointers named *_host are host memory owned by the caller; the library
 *     copies them in or out on the model's stream and synchronises before it
 *     returns.  Device memory (weights, KV cache, activations) is owned by the
 *     model and freed by mg_model_destroy.
 *   - Not re-entrant per model handle (the reference's `llm` dict is not either,
 *     src/py/mogemma/model.py:341-345); different handles may be used from
 *     different host threads.
 *
 * Reference interfaces replaced (paths inside the cofin/mogemma project):
 *   mg_model_create   <- init_model_mojo          src/mo/mogemma/core.mojo:274-364
 *   mg_model_info     <- the init_model dict keys  src/mo/mogemma/core.mojo:350-364
 *   mg_set_pos        <- llm["pos"] = 0            src/py/mogemma/model.py:341-342
 *   mg_step           <- step_mojo                 src/mo/mogemma/core.mojo:366-461
 *                        + _sample_next_token      src/py/mogemma/model.py:103-150
 *   mg_prefill        <- the prefill step loop     src/py/mogemma/model.py:344-345
 *   mg_generate       <- the decode step loop      src/py/mogemma/model.py:354-371
 *   mg_sample         <- _sample_next_token        src/py/mogemma/model.py:103-150
 *   mg_embed          <- generate_embeddings_mojo  src/mo/mogemma/core.mojo:463-600
 */
#ifndef MOGEMMA_B200_H
#define MOGEMMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MG_ABI_VERSION 1

typedef enum mg_status {
    MG_OK = 0,
    MG_ERR_INVALID = 1,      /* bad argument or inconsistent weights */
    MG_ERR_CUDA = 2,         /* a CUDA runtime call failed */
    MG_ERR_OOM = 3,          /* device allocation failed */
    MG_ERR_SEQ_EXCEEDED = 4, /* pos >= capacity: "Sequence length exceeded" */
    MG_ERR_TIMEOUT = 5,      /* a bounded device-side wait expired (kernel returned early) */
    MG_ERR_UNSUPPORTED = 6,  /* configuration not built into this library */
    MG_ERR_NCCL = 7          /* a collective failed or timed out */
} mg_status;

typedef enum mg_dtype {
    MG_F32 = 0,
    MG_BF16 = 1,
    MG_F16 = 2,
    MG_I32 = 3,
    MG_U8 = 4,
    MG_OTHER = 99
} mg_dtype;

/* One weight tensor as the reference loader hands it over: a borrowed host
 * pointer into the safetensors mmap plus shape (src/py/mogemma/loader.py:86-107).
 * Names are the HF names listed in core.mojo:79-104. */
typedef struct mg_tensor_desc {
    const char *name;
    const void *data;
    int64_t shape[4];
    int32_t ndim;
    int32_t dtype; /* mg_dtype of `data` */
} mg_tensor_desc;

typedef struct mg_options {
    int32_t struct_size;      /* sizeof(mg_options) */
    int32_t device;           /* CUDA device ordinal */
    int32_t mode;             /* 0: reference semantics; 1: gemma3 (window + dual theta) */
    int32_t weight_dtype;     /* device storage of projection weights: MG_F32 or MG_BF16 */
    int32_t max_batch;        /* decode rows held in the KV cache */
    int32_t capacity;         /* KV positions per row (reference: 8192, core.mojo:328) */
    int32_t sliding_window;   /* gemma3 mode: local-layer window */
    int32_t global_every;     /* gemma3 mode: layer l is global iff (l+1) % global_every == 0 */
    float rope_theta_local;   /* gemma3 mode */
    float rope_theta_global;  /* gemma3 mode */
    uint64_t seed;            /* sampler Philox seed */
    void *stream;             /* cudaStream_t to run on; NULL: the library creates one */
    int32_t decode_path;      /* 0: persistent decode kernel; 1: one launch per phase */
    int32_t tp_rank;          /* tensor-parallel rank (0 when tp_size == 1) */
    int32_t tp_size;          /* tensor-parallel degree (1..8); one process per GPU, see mg_tp_connect */
    int32_t prefill_path;     /* 0: mg_prefill feeds tokens one step at a time through the decode kernel (the
                                 reference's arithmetic); 1: all prompt tokens per layer at once, projections
                                 as tcgen05 GEMMs on bf16-rounded inputs (tp_size 1) */
    const void *reserved1;
    /* Device-generated weights, for benchmarks of models larger than host memory
     * (no counterpart in the reference, which reads every tensor from its
     * checkpoint): when synthetic_std > 0, every tensor whose data pointer is NULL
     * is filled on the device with N(0, synthetic_std) values from a counter-based
     * generator keyed by (synthetic_seed, tensor name, element index); lm_head.weight
     * uses the embedding's key (tied).  Read only when struct_size covers them. */
    float synthetic_std;
    int32_t reserved2;
    uint64_t synthetic_seed;
} mg_options;

typedef struct mg_model_info {
    int32_t num_layers, num_heads, num_kv_heads, head_dim;
    int32_t hidden_size, intermediate_size, vocab_size, max_seq_len;
    int32_t max_batch, mode, weight_dtype, tp_size;
    int64_t weight_bytes_per_step; /* projection + lm_head bytes streamed per decode step */
    int64_t kv_bytes_per_pos;      /* K+V bytes per cached position, all layers, one row */
    int32_t num_sms, persistent_ctas;
} mg_model_info;

/* Sampling controls of GenerationConfig (src/py/mogemma/config.py:63-69).
 * temperature/top_p are doubles because the reference divides float64 logits
 * by the Python float (model.py:105,113). */
typedef struct mg_sampling {
    double temperature; /* <= 0: greedy argmax (first maximum) */
    int32_t top_k;      /* 0 or >= vocab: no top-k filter */
    int32_t reserved0;
    double top_p;       /* (0,1): nucleus filter; otherwise off */
    const double *uniforms_host; /* optional [batch] draw variates in [0,1); NULL: Philox stream */
} mg_sampling;

typedef struct mg_model mg_model;

/* ---- library ---- */
const char *mg_last_error(void);
int32_t mg_abi_version(void);

/* ---- model lifetime ---- */
mg_status mg_model_create(const mg_tensor_desc *descs, int32_t n, const mg_options *opt, mg_model **out);
mg_status mg_model_info_get(const mg_model *m, mg_model_info *info);
mg_status mg_model_destroy(mg_model *m);
/* The cudaStream_t the model runs on (for event timing by the caller). */
void *mg_model_stream(const mg_model *m);
/* Rows one persistent decode launch holds for this model: the input stage of
 * the widest projection (down_proj: intermediate_size floats per row) must fit
 * in shared memory beside the weight ring, so it is at most 8 and fewer for
 * wide FFNs (5 for Gemma3-1B fp32).  Steps with more rows run as few launches
 * as this allows, of equal size.  0 for a NULL model. */
int32_t mg_rows_per_launch(const mg_model *m);

/* ---- positions (per batch row) ---- */
mg_status mg_set_pos(mg_model *m, int32_t row, int32_t pos); /* row -1: every row */
mg_status mg_get_pos(const mg_model *m, int32_t *pos_host, int32_t n);

/* ---- decode ----
 * One forward step for rows [0, batch): feeds token_ids_host[b] at that row's
 * position, writes its K/V, advances its position.  logits_host (nullable) gets
 * [batch, vocab] fp32 logits; sampled_host (nullable, needs s) gets one token per
 * row drawn by the _sample_next_token rules. */
mg_status mg_step(mg_model *m, const int32_t *token_ids_host, int32_t batch, float *logits_host,
                  int32_t *sampled_host, const mg_sampling *s);
/* Prefill: for each row b, feeds lens_host[b] tokens (row-major, stride max_len)
 * without computing logits, exactly like the reference's prefill loop that
 * discards step() outputs.  Positions advance by lens_host[b]. */
mg_status mg_prefill(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                     int32_t max_len);
/* Device-resident decode loop: n_steps steps; each step's input is the previous
 * step's sampled token (the first step uses the token set by the last mg_step /
 * mg_set_tokens).  tokens_host (nullable) receives [n_steps, batch] ids after the
 * loop; with NULL nothing is copied back. */
mg_status mg_generate(mg_model *m, int32_t n_steps, int32_t batch, const mg_sampling *s, int32_t *tokens_host);
mg_status mg_set_tokens(mg_model *m, const int32_t *token_ids_host, int32_t batch);

/* ---- sampling over caller logits ---- */
mg_status mg_sample(const float *logits_host, int32_t batch, int32_t vocab, const mg_sampling *s, uint64_t seed,
                    uint64_t offset, int32_t *out_host);

/* ---- sampling over device logits without allocating (no counterpart in the
 * reference, whose sampler is numpy on the host) ----
 * For callers that own all device memory through their own pool and must not
 * see cudaMalloc/cudaFree in their steady state (those calls synchronise the
 * whole device).  Draws one token per row of logits_dev ([batch] rows of
 * `vocab` floats, row stride `ld`, device memory) into out_dev (device memory),
 * asynchronously on `stream` (a cudaStream_t; NULL: the legacy default stream),
 * with the rules and the Philox stream of mg_sample: same arguments, same
 * tokens.  uniforms_dev (nullable) is a device array of [batch] variates.
 * Limits: batch <= MG_SAMPLE_STATIC_MAX_ROWS, and temperature <= 0 or
 * 0 < top_k <= 64 (MG_ERR_INVALID / MG_ERR_UNSUPPORTED beyond).  Its only
 * scratch is a static device array of 8 * 148 * 64 candidate keys (606,208
 * bytes) shared by every call on a device: calls that overlap on the GPU race;
 * calls on one stream are safe.  Every call resolves the array's address and
 * a kernel attribute on the current device (nothing is cached, so a context
 * recreated by cudaDeviceReset is picked up); the first call on a device loads
 * the kernels there: make it before any stream capture. */
#define MG_SAMPLE_STATIC_MAX_ROWS 8
#define MG_SAMPLE_STATIC_MAX_SLICES 148
mg_status mg_sample_static(const float *logits_dev, int64_t ld, int32_t batch, int32_t vocab, double temperature,
                           int32_t top_k, double top_p, const double *uniforms_dev, uint64_t seed, uint64_t offset,
                           int32_t *out_dev, void *stream);

/* ---- embeddings ----
 * Mean of final-normed hidden states per sequence (forward_sequence,
 * layers.mojo:292-370), ids row-major [batch, max_len] with lens_host[b] valid. */
mg_status mg_embed(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                   int32_t max_len, float *out_host);

/* ---- bidirectional encoder embeddings (no counterpart in the reference, whose
 * generate_embeddings is the causal mean above; an EmbeddingGemma-style
 * encoder) ----
 * Every token attends to every token of its sequence; the final-normed states
 * are mean-pooled over the row's lens_host[b] tokens, passed through the
 * optional dense head (tensors embed_head.dense0.weight [d, hidden] and
 * embed_head.dense1.weight [hidden, d]) and L2-normalised into out_host
 * [batch, hidden].  Needs a model created with prefill_path 1 (projections on
 * the tensor cores, bf16 inputs); rows go through max_batch at a time.  The
 * model's KV cache may be overwritten (head dims other than 64/128/256 run
 * the attention from the cache): treat its decode state as lost. */
mg_status mg_encode(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                    int32_t max_len, float *out_host);

/* ---- failure-detection test hooks (no counterpart in the reference, whose
 * engine has no device waits) ----
 * wait_budget_ns: budget of every bounded wait of the decode kernel (0: the
 * default of 2 s).  stall_phase: a phase whose outputs one CTA withholds (-1:
 * none; phase 5 * layer + {0 QKV, 1 attention, 2 o_proj, 3 gate/up, 4 down},
 * 5 * layers the lm_head): the waits on them run out, the kernel records the
 * site, fast-forwards to its end, and the call returns MG_ERR_TIMEOUT with the
 * model's positions restored and the model usable.  Production callers leave
 * both unset. */
mg_status mg_set_debug(mg_model *m, uint64_t wait_budget_ns, int32_t stall_phase);

/* ---- inspection (tests) ---- */
mg_status mg_read_kv(const mg_model *m, int32_t layer, int32_t row, int32_t pos, float *k_host, float *v_host);

/* ---- timeline (profiling; no reference counterpart: the reference only has
 * OpenTelemetry spans around whole calls, src/py/mogemma/telemetry.py) ----
 * When enabled, every decode launch records %globaltimer stamps per CTA and
 * phase: [ctas][phases][10] (start, ready, first tile, end, producer start,
 * producer end, then for attention phases: q/k/v loaded, normed and rotated,
 * tiles done, partial written) followed by [ctas][2] kernel begin/end.  mg_trace_read copies
 * the stamps of the most recent launch; *n_out receives the element count. */
mg_status mg_trace_enable(mg_model *m, int32_t on);
mg_status mg_trace_read(mg_model *m, uint64_t *out_host, int64_t capacity, int64_t *n_out);

/* ---- tensor parallelism (no counterpart in the reference, which runs one
 * CPU thread; the sharding follows the Gemma layout: q heads and the kv heads
 * they use, o_proj and down_proj split along their inputs, gate/up along their
 * outputs, lm_head along the vocabulary) ----
 * A model created with tp_size = T > 1 holds rank tp_rank's shard.  Its decode
 * kernel exchanges the o_proj / down_proj partial sums and the lm_head top-k
 * candidates through the other ranks' exchange buffers (peer memory over
 * NVLink) inside the same launch.  Before the first step every rank exports its
 * buffer's IPC handle, the caller gathers the T handles in rank order (for
 * example with torch.distributed over NCCL) and passes them to mg_tp_connect.
 * All ranks must then issue the same sequence of steps. */
#define MG_TP_HANDLE_BYTES 64
mg_status mg_tp_ipc_handle(const mg_model *m, void *out /* MG_TP_HANDLE_BYTES */);
mg_status mg_tp_connect(mg_model *m, const void *handles /* n * MG_TP_HANDLE_BYTES, rank order */, int32_t n);
/* ---- tensor-core GEMM (no counterpart in the reference: its projections are
 * one-token vec_mat_mul, ops.mojo:69-95; this is the dense contraction of the
 * batched prefill path) ----
 * C[M][N] (fp32, row stride ldc) = A[M][K] . B[N][K]^T with A and B bf16 device
 * matrices (row strides lda, ldb; rows 16-byte aligned), K a multiple of 64, on
 * tcgen05 tensor cores with fp32 accumulation.  err_dev is a device word that
 * receives a nonzero code if a bounded wait inside the kernel expires.
 * Asynchronous on `stream` (a cudaStream_t; NULL: the legacy default stream). */
mg_status mg_gemm_bf16(const void *a_dev, int64_t lda, const void *b_dev, int64_t ldb, float *c_dev, int64_t ldc,
                       int32_t M, int32_t N, int32_t K, uint32_t *err_dev, void *stream);

/* Unmaps the other ranks' buffers.  Every rank calls it (after its last step)
 * before any rank destroys its model, so no buffer is freed while mapped. */
mg_status mg_tp_disconnect(mg_model *m);

/* ---- Gemma 3n ("nano") decode ----
 * The reference switches to its nano graph when the checkpoint has AltUp
 * routers (src/mo/mogemma/core.mojo:26-31) and runs forward_nano_step
 * (src/mo/mogemma/layers.mojo:959-1004) per token.  mg_nano_create takes the
 * tensors the reference's nano loader reads (core.mojo:111-165: embedding,
 * final norm, lm_head, per_layer_embed{,.projection,.norm},
 * altup.{projection,unembed}.i, and per layer the base, altup, laurel and
 * per_layer_map tensors), fp32 or bf16 (widened to fp32), and a position
 * capacity.  Dimensions, the AltUp stream count and the KV-sharing start are
 * inferred as init_model_mojo does (core.mojo:296-312, 261-273).  One decode
 * step is a CUDA graph replayed per token. */
typedef struct mg_nano mg_nano;
typedef struct mg_nano_info {
    int32_t num_layers, num_heads, num_kv_heads, head_dim;
    int32_t hidden_size, intermediate_size, vocab_size, per_layer_dim;
    int32_t modalities, laurel_rank, kv_share_start, max_seq_len;
} mg_nano_info;
mg_status mg_nano_create(const mg_tensor_desc *descs, int32_t n, int32_t device, int32_t capacity, mg_nano **out);
mg_status mg_nano_info_get(const mg_nano *m, mg_nano_info *info);
mg_status mg_nano_destroy(mg_nano *m);
mg_status mg_nano_set_pos(mg_nano *m, int32_t pos);
mg_status mg_nano_get_pos(const mg_nano *m, int32_t *pos);
/* step_mojo for arch "nano" (core.mojo:366-461): the token at the model's
 * position, logits_host (nullable: no lm_head) gets [vocab] fp32 logits,
 * the position advances; MG_ERR_SEQ_EXCEEDED at capacity. */
mg_status mg_nano_step(mg_nano *m, int32_t token_id, float *logits_host);
/* The prefill loop of model.py:344-345 (steps without logits). */
mg_status mg_nano_prefill(mg_nano *m, const int32_t *ids, int32_t n);
/* forward_nano_sequence (layers.mojo:1007-1063): mean of the final hidden
 * states of tokens 0..n-1 (the model's KV rows 0..n-1 serve as scratch; its
 * position is restored). */
mg_status mg_nano_embed(mg_nano *m, const int32_t *ids, int32_t n, float *out_host);

#ifdef __cplusplus
}
#endif
#endif

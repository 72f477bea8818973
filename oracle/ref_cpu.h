/*
 * ref_cpu.h -- CPU restatement of the MoGemma Mojo engine (TEST INFRASTRUCTURE).
 *
 * This is the oracle: a plain-C, fp32, op-by-op restatement of the reference
 * engine's standard (non-nano) path, used only by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg as the checker.
 * It is never linked into, called by, or shipped as the product path.
 *
 * Reference files followed (paths inside the cofin/mogemma project):
 *   src/mo/mogemma/ops.mojo       geglu 5-30, rope_rotate 33-66, vec_mat_mul 69-95,
 *                                 rms_norm 98-136, softmax 139-182
 *   src/mo/mogemma/layers.mojo    forward_attention 16-97, forward_mlp 101-118,
 *                                 forward_layer 174-220, forward_step 224-288,
 *                                 forward_sequence 292-370
 *   src/mo/mogemma/core.mojo      init_model_mojo 274-364 (dims, KV, RoPE tables),
 *                                 step_mojo 366-461, generate_embeddings_mojo 463-600
 *
 * Extension (no reference counterpart, "gemma3" mode): per-layer sliding window
 * (global layer iff (layer+1) % global_every == 0) and separate local/global RoPE
 * theta.  In "ref" mode every layer is global and both thetas are 10000.
 *
 * Parity status: pinned against the reference's own known-answer tests
 * (src/mo/tests/test_ops.mojo, src/mo/tests/test_layers.mojo) -- see
 * tests/test_oracle_golden.py.  Mojo's SIMD reduce_add order is restated as a
 * halving tree; its exact bit order is not observable without Mojo, so
 * end-to-end comparisons use tolerances.
 */
#ifndef MG_REF_CPU_H
#define MG_REF_CPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- op level (ops.mojo) ---- */
void ref_geglu(float *out, const float *gate, const float *up, int64_t size, int nelts);
void ref_rope_rotate(float *vec, const float *cos_t, const float *sin_t, int64_t head_dim, int nelts);
void ref_vec_mat_mul(float *out, const float *x, const float *w, int64_t in_dim, int64_t out_dim, int nelts);
void ref_rms_norm(float *out, const float *x, const float *w, int64_t size, float eps, int nelts);
void ref_softmax(float *vec, int64_t size, int nelts);
void ref_rope_tables(float *cos_t, float *sin_t, int64_t max_seq_len, int64_t head_dim, float base);

/* ---- model level (layers.mojo / core.mojo) ---- */
typedef struct ref_layer_w {
    const float *input_layernorm, *post_attention_layernorm;
    const float *q_proj, *k_proj, *v_proj, *o_proj;
    const float *gate_proj, *up_proj, *down_proj;
    const float *q_norm, *k_norm; /* may be NULL (reference skips QK-norm then) */
    const float *pre_feedforward_layernorm, *post_feedforward_layernorm;
} ref_layer_w;

typedef struct ref_model ref_model;

/* mode: 0 = reference semantics, 1 = gemma3 extension (window + dual theta). */
ref_model *ref_model_create(const float *embed, const float *final_norm, const float *lm_head,
                            const ref_layer_w *layers, int32_t num_layers,
                            int64_t hidden, int64_t num_heads, int64_t num_kv_heads,
                            int64_t head_dim, int64_t intermediate, int64_t vocab,
                            int64_t max_seq_len, int32_t mode, int32_t sliding_window,
                            int32_t global_every, float theta_local, float theta_global);
void ref_model_destroy(ref_model *m);
int64_t ref_model_pos(const ref_model *m);
void ref_model_set_pos(ref_model *m, int64_t pos);
/* One decode step (step_mojo + forward_step): writes vocab logits, pos += 1.
 * Returns 0, or -1 when pos >= max_seq_len ("Sequence length exceeded"). */
int ref_step(ref_model *m, int32_t token_id, float *logits_out);
/* Same step without the lm_head projection (prefill tokens whose logits are
 * discarded by the caller, model.py:344-345).  Final hidden state is kept. */
int ref_step_no_logits(ref_model *m, int32_t token_id);
/* forward_sequence over one sequence.  ref_compat = 1 reproduces the reference
 * scratch layout exactly (including its accumulator aliasing); 0 computes the
 * mean of final-normed states that the reference intends. */
void ref_embed_sequence(ref_model *m, const int32_t *ids, int64_t seq_len, float *out, int ref_compat);
/* Bidirectional encoder (EmbeddingGemma-style extension, no reference
 * counterpart): every token attends to the whole sequence; mean of final-normed
 * states, optional dense head d0 [d0_out][hidden] then d1 [hidden][d0_out], L2
 * normalised into out [hidden].  Returns 0, or -1 for n outside [1, max_seq_len]. */
int ref_encode_sequence(ref_model *m, const int32_t *ids, int64_t n, const float *d0, int64_t d0_out,
                        const float *d1, float *out);
/* Read back KV cache rows: [layer][pos][kv_head][head_dim] (reference layout). */
const float *ref_model_k_cache(const ref_model *m);
const float *ref_model_v_cache(const ref_model *m);

/* Layer-level entry points with caller-supplied tables/cache, for replaying the
 * reference's layer known-answer tests (src/mo/tests/test_layers.mojo). */
void ref_forward_attention_raw(float *out, const float *x, const ref_layer_w *w, int64_t pos, int64_t hidden,
                               int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, const float *cos_t,
                               const float *sin_t, float *k_cache, float *v_cache, float *scratch);
void ref_forward_mlp_raw(float *out, const float *x, const ref_layer_w *w, int64_t hidden, int64_t intermediate,
                         float *scratch);
void ref_forward_layer_raw(float *out, const float *x, const ref_layer_w *w, int64_t pos, int64_t hidden,
                           int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, int64_t intermediate,
                           const float *cos_t, const float *sin_t, float *k_cache, float *v_cache, float *scratch);

/* Threads used by vec_mat_mul's row loop (1 = the reference's single thread). */
void ref_set_threads(int n);
int ref_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif

// decode.cuh -- parameter block and constants of the persistent decode kernel.
//
// One launch runs a contiguous range of "phases" of a decode step for B rows:
//   per layer l: QKV(l), ATT(l), O(l), GU(l), D(l); then LMH, then SAMPLE.
// Each CTA is split into 8 consumer warps and 1 producer warp.  The producer
// streams this CTA's weight tiles (and past K/V rows) through a ring of
// shared-memory stages with 1-D bulk async copies, running ahead across phase
// boundaries because weights never depend on activations.  Consumers poll the
// previous phase's activations, which are stored as tagged words (value and
// the tag of the forward and layer that wrote it, in one 64-bit store).
#pragma once

#include <stdint.h>

namespace mg {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kStageBytes = 36864;   // one ring stage
constexpr int kMaxRows = 8;          // batch rows per persistent launch
constexpr int kMaxTp = 8;            // tensor-parallel ranks
constexpr int kMaxBatch = 64;        // rows a model holds (more than kMaxRows: batched tensor-core steps)
constexpr int kMaxHeadDim = 256;
constexpr int kMaxQPerKv = 8;
constexpr int kMaxTopK = 64;         // fused top-k width
constexpr int kAttTile = 16;         // positions per attention tile
constexpr int kPartHead = 4;         // floats before a split-KV partial's acc: m, l, 2 pad (16-byte aligned acc)
constexpr int kSplitVals = 2 * 16 * kMaxRows;  // (gate, up) x rows of a group (<= 16) x kernel rows
constexpr int kSplitKinds = 5;          // indexed by phase kind (QKV, ATT unused, O, GU, D)
constexpr int kMaxChunks = 32;       // split-KV chunks per (row, kv head); one warp lane each in the combine
constexpr int kMaxLayers = 64;       // layers a model may have (tags hold epoch * kMaxLayers + layer)
constexpr uint32_t kMaxEpoch = (1u << 26) - 1;  // forwards before the tagged buffers are cleared and the count restarts

enum PhaseKind : int { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_D = 4, PH_LMH = 5, PH_SAMPLE = 6 };

// lm_mode
constexpr int kLmNone = 0;    // no lm_head (prefill tokens whose logits are discarded)
constexpr int kLmLogits = 1;  // logits (+ fused top-k candidates when topk > 0)
constexpr int kLmEmbed = 2;   // accumulate final-normed state into emb_acc

struct LayerPtrs {
    const void *qkv;   // [qkv_rows][Hp]   rows: q (Hq*hd), k (Hkv*hd), v (Hkv*hd)
    const void *o;     // [H][Ap]
    const void *gate;  // [I][Hp]
    const void *up;    // [I][Hp]
    const void *down;  // [H][Ip]
    const float *in_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln;  // [H]
    const float *q_norm, *k_norm;                                // [hd] or null
    int32_t is_global;
    int32_t pad_;
};

struct DecodeParams {
    // dimensions (padded row lengths are multiples of 128 elements)
    int32_t L, H, Hp, Hq, Hkv, hd, hdp, I, Ip, V, A, Ap, qkv_rows;
    int32_t B;        // rows in this launch
    int32_t cap;      // KV positions per row
    int32_t window;   // local-layer window (gemma3 mode), 0 = unbounded
    int32_t S;        // ring stages
    int32_t att_ch;   // positions per attention chunk (multiple of kAttTile)
    int32_t max_ch;   // chunks allocated per (row, kv head)
    int32_t lm_mode;
    int32_t topk;     // fused candidates per row (0: none, 1: argmax, <= kMaxTopK)
    int32_t ph_begin, ph_end;
    int32_t xs_floats;  // floats reserved for the activation stage in shared memory
    int32_t step_t;     // token index within mg_prefill/mg_embed (row active iff step_t < nvalid[b])
    int32_t ids_ld;
    int32_t max_inflight;  // weight/KV tiles a CTA keeps in flight (<= S); bounds memory-queue latency
    int32_t pf_tiles;      // how far (tiles) the producer prefetches into L2 ahead of its ring loads
    float inv_h;        // 1 / H

    const LayerPtrs *layers;
    const void *lm_head;   // [V][Hp]
    const void *embed;     // [V][embed_ld]
    int64_t embed_ld;
    const float *final_norm;
    const float *rope_cos_l, *rope_sin_l, *rope_cos_g, *rope_sin_g;  // [cap][hd/2]
    float *kc, *vc;                                                   // [L][Bmax][Hkv][cap][hdp]
    int64_t kv_layer_stride, kv_row_stride, kv_head_stride;

    // activations [B][...] as tagged words (tg_pack in common.cuh): the value
    // and the tag of the (forward, layer) that wrote it.  Readers poll the words.
    // The large vectors that every CTA reads whole stay plain floats behind a
    // phase counter (doubling their bytes costs more than the counter saves).
    uint64_t *h, *r, *qkv, *o_raw, *mlp_raw;
    float *act;         // [B][Ip] GeGLU output
    float *attn_part;   // split-KV partials [B][Hkv][kMaxChunks][Gq][hd + kPartHead]
    float *logits;      // [B][V]
    uint64_t *cand_key; // [B][G][kMaxTopK] per-CTA top-k keys of the lm_head rows
    float *emb_acc;     // [B][H]

    int32_t *tok;            // [B] current input token per row
    int32_t *pos;            // [B] position of the next token per row
    const int32_t *ids;      // optional [B][ids_ld] token matrix (prefill / embed)
    const int32_t *nvalid;   // optional [B] valid tokens per row
    int32_t *out_tokens;     // optional [B] sampled tokens of this step

    // sampling
    double temperature, top_p;
    int32_t top_k_req;   // the caller's top_k (reference semantics)
    int32_t sample;      // 1: draw a token per row in PH_SAMPLE
    const double *uniforms;  // optional [B]
    uint64_t seed;
    uint64_t rng_offset;     // Philox counter of this step's draws

    uint32_t epoch;   // forward counter (from 1): words of layer l carry tag epoch * kMaxLayers + l
    uint32_t pad4_;
    uint64_t wait_ns;     // budget of every bounded wait (0: the default, kWaitBudgetNs)
    int32_t stall_phase;  // test hook: one CTA withholds its outputs of this phase (-1: none)
    int32_t att_split;    // 1: attention items per q head (head dim 256 only); 0: per kv head group
    int32_t gemv_split;   // 1: projection phases may split a row group between two CTAs (see gemv_geom)
    int32_t pad5_;
    // split row groups: partial row sums [kind][boundary G][part 2][kSplitVals] and one
    // exchange word per (kind, boundary) -- inside the tagged block, so cleared with it
    float *split_part;
    uint64_t *split_tag;
    uint32_t *sync;   // phase counters [n_phases], att_done [L], att_cnt [B*Hkv], exit [1]
    uint32_t *err;    // device error word
    int32_t n_phases;
    float inv_hd;       // 1 / head_dim
    // optional timeline: [G][n_phases][kTraceSlots] %globaltimer stamps, then [G][2] kernel begin/end
    uint64_t *trace;
    float att_scale;    // 1 / sqrt(head_dim), as the reference computes it (layers.mojo:65)
    float emb_scale;    // sqrt(H) (layers.mojo:247-251)

    // tensor parallelism (tp > 1): this rank holds q heads, kv heads, FFN rows
    // and vocabulary rows of its shard (the dimensions above are the shard's).
    // The row-split o_proj and down_proj write their partial [B][H] rows into
    // every rank's exchange buffer (peer memory over NVLink) and count on each
    // rank's exchange counters; lm_head candidates are exchanged the same way.
    int32_t tp, tp_rank;
    int32_t V_full;          // vocabulary of the whole model (token id range)
    int32_t vocab_off;       // first vocabulary row of this rank's lm_head shard
    int32_t xB;              // rows per source block in the exchange buffers (the model's max batch)
    int32_t row_base;        // model row of this launch's row 0 (launches over row groups; Philox row index)
    uint64_t xep;            // exchanges of earlier forwards: layer l exchanges index xep + l
    uint64_t lm_ep;          // candidate exchanges of earlier forwards
    char *xpeer[kMaxTp];     // exchange buffer of every rank (this rank's own at tp_rank)
    int64_t x_cnt, x_o, x_d, x_cand;  // byte offsets in an exchange buffer
};

// trace slots per (CTA, phase)
constexpr int kTraceSlots = 10;
constexpr int kTrAttLoaded = 6;   // attention: raw q/k/v in shared memory (first item)
constexpr int kTrAttRoped = 7;    // attention: QK-norm + RoPE done (first item)
constexpr int kTrAttTiles = 8;    // attention: all tiles of the first item done
constexpr int kTrAttPart = 9;     // attention: partial of the first item written
constexpr int kTrStart = 0;      // consumer reaches the phase
constexpr int kTrReady = 1;      // its input dependency is satisfied
constexpr int kTrPrologue = 2;   // input vector staged in shared memory
constexpr int kTrEnd = 3;        // phase done and signalled
constexpr int kTrProdStart = 4;  // producer starts issuing this phase's tiles
constexpr int kTrProdEnd = 5;    // producer issued its last tile of the phase

inline int num_phases(int L) { return 5 * L + 2; }

// Tile shape of a projection matrix with padded row length Kp: tiles of `rps`
// rows (8 warps x rows per warp) by `kc` columns; `mult` = 2 stores the gate
// and up rows of the same output rows together.  kc divides Kp (nseg segments
// per row) so every tile is the same size and fits one ring stage.  On the
// device a matrix is stored tile by tile -- [row group][segment][mult*rps][kc]
// -- so each tile is one contiguous bulk copy.
struct TileShape {
    int rps, mult, kc, nseg;
};
__host__ __device__ inline TileShape tile_shape(int Kp, int esz, bool pair) {
    TileShape t;
    t.rps = kConsumerWarps * (esz == 2 ? 2 : 1);
    t.mult = pair ? 2 : 1;
    const int per_row = t.rps * t.mult * esz;  // bytes per column of a tile
    int n = (Kp * per_row + kStageBytes - 1) / kStageBytes;
    if (n < 1) n = 1;
    while (Kp % n != 0 || (Kp / n) % 8 != 0) ++n;
    t.nseg = n;
    t.kc = Kp / n;
    return t;
}
// Elements of one tile, and of a tiled matrix with N rows.
__host__ __device__ inline int64_t tile_elems(const TileShape &t) {
    return static_cast<int64_t>(t.mult) * t.rps * t.kc;
}
__host__ __device__ inline int64_t tiled_elems(const TileShape &t, int64_t N) {
    return (N + t.rps - 1) / t.rps * t.nseg * tile_elems(t);
}

}  // namespace mg

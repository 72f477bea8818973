// decode_kernel.cuh -- persistent sm_100a decode kernel for the Gemma 3 forward step.
//
// Restates, for B rows at once, forward_step (src/mo/mogemma/layers.mojo:224-288)
// with forward_layer (174-220), forward_attention (16-97) and forward_mlp
// (101-118), plus the token draw of _sample_next_token (src/py/mogemma/model.py:
// 103-150).  Layout and scheduling are this library's own:
//
//  * Every projection is a GEMV phase whose rows are split evenly over the CTAs
//    (one CTA per SM).  Weight rows are padded to 128 elements on the device.
//  * Warp 8 of each CTA is a producer: one lane walks the CTA's tile schedule
//    for the whole launch and streams weight tiles (and cached K/V rows for
//    attention) into a ring of shared-memory stages with cp.async.bulk, ahead
//    of the consumers and across phase boundaries (weights never depend on
//    activations).
//  * Warps 0-7 consume: each phase polls its input activations -- tagged
//    words (value + tag of the forward and layer that wrote it, one 64-bit
//    store) written by every CTA in the previous phase -- until each carries
//    the expected tag, builds the normalised input vector in shared memory
//    (RMSNorm with (1 + w), residual adds), then multiplies it by the staged
//    tiles with 128-bit shared loads and warp-shuffle reductions.  Polling the
//    data itself replaces a counter, its release fence and a second load
//    round trip per hand-off (measured 1.2 us instead of 2.0 us).  Norm
//    weights and RoPE rows are loaded before the poll.
//  * Fusions: input/pre-ff/post-attn/post-ff/final norms and residual adds in
//    the next phase's prologue; QK-norm, RoPE and the K/V write in the attention
//    prologue; GeGLU in the gate/up epilogue; the split-KV combine in the
//    o_proj prologue; a per-CTA top-k of the lm_head rows in its epilogue; the
//    draw in the last phase.
//  * All waits are bounded (common.cuh); on timeout the kernel fast-forwards.
//  * The batch row count NB is a template parameter of the whole kernel: a
//    launch for B rows runs code sized for exactly B rows.  Loops over rows
//    sized for the largest batch cost the batch-1 decode about 2.5 us per norm
//    prologue (measured), so each row count is its own instantiation, compiled
//    in its own translation unit (decode_nb<N>.cu).
#pragma once
#include "common.cuh"
#include "decode.cuh"
#include "select.cuh"

namespace mg {

// The launch's budget for every bounded wait (ns of %globaltimer), set by thread
// 0 from DecodeParams::wait_ns before the first wait.
__shared__ uint64_t g_wait_ns;

// ---------------------------------------------------------------- sync layout
__device__ __forceinline__ uint32_t *ctr_phase(const DecodeParams &p, int ph) { return p.sync + ph; }
__device__ __forceinline__ uint32_t *ctr_exit(const DecodeParams &p) { return p.sync + p.n_phases; }

__device__ __forceinline__ void phase_of(int ph, int L, int &kind, int &layer) {
    if (ph < 5 * L) {
        layer = ph / 5;
        kind = ph - 5 * layer;
    } else if (ph == 5 * L) {
        kind = PH_LMH;
        layer = L - 1;
    } else {
        kind = PH_SAMPLE;
        layer = L - 1;
    }
}

// Rotating slot so the CTAs that get one extra row differ from phase to phase.
__device__ __forceinline__ int cta_slot(int ph) { return static_cast<int>((blockIdx.x + 61u * ph) % gridDim.x); }

// A CTA's share of a projection phase, as a schedule of row groups:
//   whole groups [full_g0, full_g0 + nfull) (= row0, nrows, ngroups, tiles),
//   all segments; then, with a split, the tail of group lead_g (segments
//   [lead_s0, nseg)), whose head the previous slot computes, and the head of
//   group tail_g (segments [0, tail_s1)), whose tail the next slot computes.
// The two CTAs of a split group exchange partial row sums; the second to
// arrive adds them and writes the rows (gemv_split_rows).
template <typename WT>
struct GemvGeom {
    const WT *tiles;  // this CTA's first tile (tiled layout, see tile_shape)
    const WT *base;   // tile (group 0, segment 0) of the matrix
    bool pair;        // gate/up phase: each tile holds gate rows then up rows
    bool split;       // the schedule holds split groups
    int64_t row0;     // first output row of this CTA (whole-group schedules)
    int nrows;        // output rows of this CTA (the last group may be partial)
    int N;            // output rows of the matrix
    int Kp, kc, nseg, rps, ngroups;
    int tile_elems;
    int kind, slot, layer;
    int full_g0, nfull;
    int lead_g, lead_s0;  // lead_g < 0: none
    int tail_g, tail_s1;  // tail_g < 0: none
    // split piece k (0: the lead group's tail, 1: the tail group's head); false if absent
    __device__ __forceinline__ bool split_piece(int k, int &grp, int &s0, int &s1) const {
        grp = k == 0 ? lead_g : tail_g;
        s0 = k == 0 ? lead_s0 : 0;
        s1 = k == 0 ? nseg : tail_s1;
        return grp >= 0;
    }
};

template <typename WT>
__device__ __forceinline__ void gemv_geom(const DecodeParams &p, const LayerPtrs &lp, int kind, int ph,
                                          GemvGeom<WT> &g) {
    int N;
    const WT *base;
    g.pair = false;
    switch (kind) {
        case PH_QKV:
            N = p.qkv_rows;
            g.Kp = p.Hp;
            base = static_cast<const WT *>(lp.qkv);
            break;
        case PH_O:
            N = p.H;
            g.Kp = p.Ap;
            base = static_cast<const WT *>(lp.o);
            break;
        case PH_GU:
            N = p.I;
            g.Kp = p.Hp;
            base = static_cast<const WT *>(lp.gate);
            g.pair = true;
            break;
        case PH_D:
            N = p.H;
            g.Kp = p.Ip;
            base = static_cast<const WT *>(lp.down);
            break;
        default:
            N = (p.lm_mode == kLmLogits) ? p.V : 0;
            g.Kp = p.Hp;
            base = static_cast<const WT *>(p.lm_head);
            break;
    }
    const TileShape ts = tile_shape(g.Kp, static_cast<int>(sizeof(WT)), g.pair);
    g.rps = ts.rps;
    g.kc = ts.kc;
    g.nseg = ts.nseg;
    g.tile_elems = static_cast<int>(tile_elems(ts));
    // row groups are split evenly over the CTAs, rotating the remainder by phase
    const int groups = (N + g.rps - 1) / g.rps;
    const int slot = cta_slot(ph);
    const int g0 = static_cast<int>(static_cast<int64_t>(groups) * slot / gridDim.x);
    const int g1 = static_cast<int>(static_cast<int64_t>(groups) * (slot + 1) / gridDim.x);
    g.ngroups = g1 - g0;
    g.row0 = static_cast<int64_t>(g0) * g.rps;
    g.nrows = static_cast<int>(min(static_cast<int64_t>(N), static_cast<int64_t>(g1) * g.rps) - g.row0);
    if (g.nrows < 0) g.nrows = 0;
    g.tiles = base + static_cast<int64_t>(g0) * g.nseg * g.tile_elems;
    // The host marks the phase kinds whose whole groups leave some CTAs two or
    // more tiles above the even share (split_kinds, engine.cu); their (group,
    // segment) tiles are split evenly instead.  Every slot then holds at least
    // nseg tiles, so a group is shared by two slots at most.
    // (bf16 weights only: the fp32 kernels compile without it, exactly as before it existed)
    g.split = sizeof(WT) == 2 && ((p.gemv_split >> kind) & 1);
    if constexpr (sizeof(WT) != 2) return;
    if (g.split) {
        const int G = static_cast<int>(gridDim.x);
        const int U = groups * g.nseg;
        g.N = N;
        g.base = base;
        g.kind = kind;
        g.slot = slot;
        int k2;
        phase_of(ph, p.L, k2, g.layer);
        g.lead_g = g.tail_g = -1;
        g.lead_s0 = g.tail_s1 = 0;
        const int u0 = U * slot / G, u1 = U * (slot + 1) / G;
        const int ga = u0 / g.nseg, sa = u0 - ga * g.nseg;
        const int gb = u1 / g.nseg, sb = u1 - gb * g.nseg;
        g.full_g0 = sa ? ga + 1 : ga;
        g.nfull = gb - g.full_g0;
        if (sa) {
            g.lead_g = ga;
            g.lead_s0 = sa;
        }
        if (sb) {
            g.tail_g = gb;
            g.tail_s1 = sb;
        }
        // the whole-group fields describe the full groups (streamed first)
        g.ngroups = g.nfull;
        g.row0 = static_cast<int64_t>(g.full_g0) * g.rps;
        g.nrows = static_cast<int>(min(static_cast<int64_t>(N), static_cast<int64_t>(gb) * g.rps) - g.row0);
        if (g.nrows < 0) g.nrows = 0;
        g.tiles = base + static_cast<int64_t>(g.full_g0) * g.nseg * g.tile_elems;
    }
}

// Attention work split: items are (row, unit, chunk of att_ch positions), a
// unit being a kv head with its q heads, or (att_split) a single q head --
// four times the items for Gemma3-1B's 4 q heads per kv head, each a quarter
// of the work, so the phase ends sooner when CTAs are idle anyway.
struct AttRows {
    int lo[kMaxRows], nch[kMaxRows];
    int nitems;
};

template <int NB>
__device__ __forceinline__ void att_rows(const DecodeParams &p, bool global, const int *s_pos, AttRows &a) {
    a.nitems = 0;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        {
            const int pos = s_pos[b];
            int lo = 0;
            if (!global && p.window > 0 && pos - p.window + 1 > 0) lo = pos - p.window + 1;
            a.lo[b] = lo;
            a.nch[b] = (pos + 1 - lo + p.att_ch - 1) / p.att_ch;
            a.nitems += (p.att_split ? p.Hq : p.Hkv) * a.nch[b];
        }
    }
}

// Item -> row b, kv head kvh, chunk c, and the item's first q head qh0 (all of
// the kv head's q heads, or the one q head of an att_split item).
__device__ __forceinline__ void att_item(const DecodeParams &p, const AttRows &a, int item, int &b, int &kvh,
                                         int &c, int &qh0) {
    const int units = p.att_split ? p.Hq : p.Hkv;
    int base = 0;
    b = 0;
    for (; b < p.B - 1; ++b) {
        const int cnt = units * a.nch[b];
        if (item < base + cnt) break;
        base += cnt;
    }
    const int r = item - base;
    const int u = r / a.nch[b];
    c = r - u * a.nch[b];
    const int Gq = p.Hq / p.Hkv;
    kvh = p.att_split ? u / Gq : u;
    qh0 = p.att_split ? u : u * Gq;
}

__device__ __forceinline__ float *att_part(const DecodeParams &p, int b, int kvh, int c) {
    const int Gq = p.Hq / p.Hkv;
    return p.attn_part + ((static_cast<int64_t>(b) * p.Hkv + kvh) * kMaxChunks + c) * Gq * (p.hd + kPartHead);
}

// Tag of the words written for `layer` in this forward.
__device__ __forceinline__ uint32_t tag_of(const DecodeParams &p, int layer) {
    return p.epoch * static_cast<uint32_t>(kMaxLayers) + static_cast<uint32_t>(layer);
}

// ---------------------------------------------------------------- shared memory
struct Smem {
    uint64_t *full;
    uint64_t *empty;
    unsigned char *ring;
    float *xs;  // activation stage / attention scratch / selection scratch
    LayerPtrs *layers;
};

struct SmallSmem {
    float *xdst_o[kMaxTp];  // tensor parallelism: this rank's receive block on every rank (o_proj)
    float *xdst_d[kMaxTp];  // (down_proj)
    AttRows att;    // consumers' split of the current attention phase
    AttRows att_p;  // the producer's (it runs phases ahead)
    int pos[kMaxRows];
    int tok[kMaxRows];
    int active[kMaxRows];
    float red[kConsumerWarps * kMaxRows * 4];
    uint32_t flag;
    uint32_t split_second;  // gemv_split_rows: this CTA completes the split group
    uint64_t *tr_ready;  // trace slots of the current phase (consumer thread 0 only)
    uint64_t *tr_end;
};

// Optional timeline stamp (see kTraceSlots); null trace pointer = off.
__device__ __forceinline__ uint64_t *trace_slot(const DecodeParams &p, int ph, int slot) {
    return p.trace ? p.trace + (static_cast<size_t>(blockIdx.x) * p.n_phases + ph) * kTraceSlots + slot : nullptr;
}
__device__ __forceinline__ void trace_mark(uint64_t *slot) {
    if (slot) *slot = globaltimer_ns();
}

// ---------------------------------------------------------------- consumer helpers
// Sum over the consumer threads of each of NB per-thread row values.
template <int NB>
__device__ __forceinline__ void block_sum_rows(float (&v)[NB], SmallSmem &ss, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const float s = warp_sum(v[b]);
        if (lane == 0) ss.red[warp * kMaxRows + b] = s;
    }
    consumer_sync(kConsumerThreads);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) t += ss.red[w * kMaxRows + b];
        v[b] = t;
    }
    consumer_sync(kConsumerThreads);
}

// Sum over the consumer threads of four per-thread values for each of NB rows.
template <int NB>
__device__ __forceinline__ void block_sum4_rows(float (&v)[4][NB], SmallSmem &ss, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float s = warp_sum(v[k][b]);
            if (lane == 0) ss.red[(warp * 4 + k) * kMaxRows + b] = s;
        }
    consumer_sync(kConsumerThreads);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) t += ss.red[(w * 4 + k) * kMaxRows + b];
            v[k][b] = t;
        }
    consumer_sync(kConsumerThreads);
}

constexpr int kNormPer = 8;  // elements per thread held in registers per chunk (H <= 2048 in one chunk)

// Norm weights of a phase prologue, loaded before its dependency wait.
struct NormW {
    float wa[kNormPer], wn[kNormPer];
};
__device__ __forceinline__ void norm_prefetch(NormW &nw, const float *w_add, const float *w_next, int H, int tid) {
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int i = tid + j * kConsumerThreads;
        nw.wa[j] = (w_add != nullptr && i < H) ? __ldg(w_add + i) : 0.f;
        nw.wn[j] = (w_next != nullptr && i < H) ? __ldg(w_next + i) : 0.f;
    }
    // Pin the loads here: without this the compiler may sink them past the
    // dependency wait, onto the prologue's critical path.
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) asm volatile("" : "+f"(nw.wa[j]), "+f"(nw.wn[j]));
}

// For rows b < NB:  x = base[b] + rmsnorm(add[b]) * (1 + w_add);  out[b] <- x
// (when out != null);  xs[b] <- rmsnorm(x) * (1 + w_next), zero padded to Kp.
// base rows ([NB][H] tagged words) and add rows (tagged words add_t, or with
// XSUM nadd per-rank float blocks add_x, add_stride floats apart, that the
// caller has already waited for and that are summed in rank order so every
// rank gets the same bits) were written by other CTAs: all loads of a chunk
// are issued before any is used, and tagged words are polled until they carry
// `tag`.  out is written with out_tag.  Returns false if a poll gave up.
template <int NB, bool XSUM = false>
__device__ __forceinline__ bool stage_norm(const uint64_t *base, const uint64_t *add_t, const float *add_x,
                                           uint32_t tag, const float *w_add, const float *w_next, const NormW &nw,
                                           uint64_t *out, uint32_t out_tag, int H, float inv_h, int Kp, float *xs,
                                           SmallSmem &ss, int tid, uint32_t *err, uint32_t site, int nadd = 1,
                                           int64_t add_stride = 0) {
    bool ok = true;
    // One block reduction: with a = add * (1 + w_add) and s the add row's RMS
    // scale, sum(x^2) = sum(base^2) + 2 s sum(base a) + s^2 sum(a^2), so the
    // four sums sum(add^2), sum(base^2), sum(base a), sum(a^2) give both scales.
    float sums[4][NB];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int b = 0; b < NB; ++b) sums[k][b] = 0.f;
    float *xb = xs + NB * Kp;  // base rows staged next to the activation stage
    for (int j0 = 0; j0 * kConsumerThreads < H; j0 += kNormPer) {
        float wa[kNormPer];
        if (j0 == 0) {
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) wa[j] = nw.wa[j];
        } else {
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int i = tid + (j0 + j) * kConsumerThreads;
                wa[j] = i < H ? __ldg(w_add + i) : 0.f;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint64_t *brow = base + static_cast<int64_t>(b) * H;
            const uint64_t *arow = add_t + static_cast<int64_t>(b) * H;
            uint64_t wb[kNormPer], wv[kNormPer];
            float v[kNormPer];
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int i = tid + (j0 + j) * kConsumerThreads;
                wb[j] = i < H ? tg_load(brow + i) : tg_pack(0.f, tag);
                if constexpr (!XSUM) wv[j] = i < H ? tg_load(arow + i) : tg_pack(0.f, tag);
            }
            if constexpr (XSUM) {
                float t[kMaxTp][kNormPer];
#pragma unroll
                for (int r = 0; r < kMaxTp; ++r)
#pragma unroll
                    for (int j = 0; j < kNormPer; ++j) {
                        const int i = tid + (j0 + j) * kConsumerThreads;
                        t[r][j] = (r < nadd && i < H)
                                      ? __ldcg(add_x + r * add_stride + static_cast<int64_t>(b) * H + i)
                                      : 0.f;
                    }
#pragma unroll
                for (int j = 0; j < kNormPer; ++j) {
                    v[j] = t[0][j];
#pragma unroll
                    for (int r = 1; r < kMaxTp; ++r)
                        if (r < nadd) v[j] += t[r][j];
                }
            }
            auto bsrc = [&](int j) { return brow + tid + (j0 + j) * kConsumerThreads; };
            ok = tg_settle(wb, tag, bsrc, err, site, g_wait_ns) && ok;
            if constexpr (!XSUM) {
                auto asrc = [&](int j) { return arow + tid + (j0 + j) * kConsumerThreads; };
                ok = tg_settle(wv, tag, asrc, err, site, g_wait_ns) && ok;
#pragma unroll
                for (int j = 0; j < kNormPer; ++j) v[j] = tg_val(wv[j]);
            }
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int i = tid + (j0 + j) * kConsumerThreads;
                const float bv = tg_val(wb[j]);
                if (i < H) {
                    xs[b * Kp + i] = v[j];
                    xb[b * H + i] = bv;
                }
                const float av = v[j] * (1.0f + wa[j]);
                sums[0][b] += v[j] * v[j];
                sums[1][b] += bv * bv;
                sums[2][b] += bv * av;
                sums[3][b] += av * av;
            }
        }
    }
    block_sum4_rows<NB>(sums, ss, tid);
    float inv_a[NB], inv_x[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        inv_a[b] = rms_inv(sums[0][b], inv_h);
        const float sx = sums[1][b] + 2.0f * inv_a[b] * sums[2][b] + inv_a[b] * inv_a[b] * sums[3][b];
        inv_x[b] = rms_inv(fmaxf(sx, 0.f), inv_h);
    }
    // x = base + add * inv_a * (1 + w_add) -> out; xs = x * inv_x * (1 + w_next), zero padded to Kp
    for (int j0 = 0; j0 * kConsumerThreads < Kp; j0 += kNormPer) {
        float wa[kNormPer], wn[kNormPer];
        if (j0 == 0) {
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                wa[j] = nw.wa[j];
                wn[j] = nw.wn[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int i = tid + (j0 + j) * kConsumerThreads;
                wa[j] = i < H ? __ldg(w_add + i) : 0.f;
                wn[j] = i < H ? __ldg(w_next + i) : 0.f;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int i = tid + (j0 + j) * kConsumerThreads;
                if (i < H) {
                    const float x = xb[b * H + i] + xs[b * Kp + i] * inv_a[b] * (1.0f + wa[j]);
                    if (out) tg_store(out + static_cast<int64_t>(b) * H + i, x, out_tag);
                    xs[b * Kp + i] = x * inv_x[b] * (1.0f + wn[j]);
                } else if (i < Kp) {
                    xs[b * Kp + i] = 0.0f;
                }
            }
        }
    }
    consumer_sync(kConsumerThreads);
    return ok;
}

// Layer 0 input: x = E[tok] * sqrt(H) (model.mojo:62-68, layers.mojo:247-251),
// out <- x, xs <- rmsnorm(x) * (1 + w).
template <typename WT, int NB>
__device__ __noinline__ void stage_embed(const WT *E, int64_t ld, const int *toks, const float *w, uint64_t *out,
                                         uint32_t out_tag, int H, float inv_h, float scale, int Kp, float *xs,
                                         SmallSmem &ss, int tid) {
    float sq[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float s = 0.f;
        for (int i = tid; i < H; i += kConsumerThreads) {
            const float x = ld_w(E + static_cast<int64_t>(toks[b]) * ld + i) * scale;
            xs[b * Kp + i] = x;
            if (out) tg_store(out + static_cast<int64_t>(b) * H + i, x, out_tag);
            s += x * x;
        }
        sq[b] = s;
    }
    block_sum_rows<NB>(sq, ss, tid);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const float inv = rms_inv(sq[b], inv_h);
        for (int i = tid; i < Kp; i += kConsumerThreads) xs[b * Kp + i] = i < H ? xs[b * Kp + i] * inv * (1.0f + w[i]) : 0.f;
    }
    consumer_sync(kConsumerThreads);
}

// Announce this CTA's part of a phase (release at gpu scope).
__device__ __forceinline__ void cta_signal(uint32_t *ctr, uint32_t n, SmallSmem &ss, int tid) {
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
        // The barrier orders every consumer's writes before thread 0's release;
        // red.release is cumulative over them at gpu scope.
        if (n) red_release_add_u32(ctr, n);
        trace_mark(ss.tr_end);
    }
}

// End of a phase whose results are tagged words (no counter to count on):
// the barrier keeps the next prologue from overwriting the shared activation
// stage while a warp still reads it.
__device__ __forceinline__ void phase_done(SmallSmem &ss, int tid) {
    consumer_sync(kConsumerThreads);
    if (tid == 0) trace_mark(ss.tr_end);
}

// Wait for a counter; uniform result across consumer threads.
__device__ __forceinline__ bool cta_wait(const uint32_t *ctr, uint32_t target, uint32_t *err, uint32_t site,
                                         SmallSmem &ss, int tid) {
    if (tid == 0) {
        ss.flag = wait_counter_geq(ctr, target, err, site, g_wait_ns) ? 1u : 0u;
        trace_mark(ss.tr_ready);
    }
    consumer_sync(kConsumerThreads);
    const bool ok = ss.flag != 0u;
    consumer_sync(kConsumerThreads);
    return ok;
}

// ---- tensor parallelism: exchange buffers and counters (see DecodeParams)
// which: 0 o_proj partials, 1 down_proj partials, 2 lm_head candidates
__device__ __forceinline__ uint64_t *xcnt(const DecodeParams &p, int rank, int which) {
    return reinterpret_cast<uint64_t *>(p.xpeer[rank] + p.x_cnt) + which;
}
__device__ __forceinline__ float *xrecv(const DecodeParams &p, int rank, int which) {
    return reinterpret_cast<float *>(p.xpeer[rank] + (which == 0 ? p.x_o : p.x_d));
}
// After a phase whose results went to every rank: count this CTA on every
// rank's counter (system scope; the stores before it are peer stores).
__device__ __forceinline__ void xsignal(const DecodeParams &p, int which, int tid) {
    if (tid == 0) {
        fence_acq_rel_sys();
        for (int r = 0; r < p.tp; ++r) red_release_sys_add_u64(xcnt(p, r, which), 1ull);
    }
}
// Wait until every CTA of every rank has counted exchange `index` of kind
// `which` (counters only grow: exchange index e completes at (e + 1) * tp * G).
__device__ __forceinline__ bool xwait(const DecodeParams &p, int which, uint64_t index, uint32_t site,
                                      SmallSmem &ss, int tid) {
    if (tid == 0) {
        const uint64_t target = (index + 1) * static_cast<uint64_t>(p.tp) * gridDim.x;
        ss.flag = wait_counter_geq_sys(xcnt(p, p.tp_rank, which), target, p.err, site, g_wait_ns) ? 1u : 0u;
        trace_mark(ss.tr_ready);
    }
    consumer_sync(kConsumerThreads);
    const bool ok = ss.flag != 0u;
    consumer_sync(kConsumerThreads);
    return ok;
}

// ---------------------------------------------------------------- GEMV consumer
// Where a GEMV phase's row results go: out[b * ld + row] = dot, or with a
// gate/up pair out[b * ld + row] = gelu_erf(gate) * up (ops.mojo:19-22), as
// tagged words (tout, tag) or plain floats (fout: logits).  With tensor
// parallelism the partial rows of o_proj / down_proj go to every rank's
// exchange buffer instead: xdst[k] is rank k's receive block of this rank (nx
// destinations, nx = 0: local out).
struct GemvOut {
    uint64_t *tout;
    float *fout;
    int64_t ld;
    uint32_t tag;
    float *const *xdst = nullptr;
    int nx = 0;
    bool mute = false;  // test hook (DecodeParams::stall_phase): the results are withheld
};
__device__ __forceinline__ GemvOut gemv_out_tagged(uint64_t *out, int64_t ld, uint32_t tag) {
    return GemvOut{out, nullptr, ld, tag};
}
__device__ __forceinline__ GemvOut gemv_out_float(float *out, int64_t ld) { return GemvOut{nullptr, out, ld, 0u}; }
__device__ __forceinline__ GemvOut gemv_out_peers(float *const *xdst, int nx, int64_t ld) {
    return GemvOut{nullptr, nullptr, ld, 0u, xdst, nx};
}
__device__ __forceinline__ void gemv_store(const GemvOut &o, int64_t idx, float v) {
    if (o.mute) return;
    if (o.nx) {
        for (int k = 0; k < o.nx; ++k) o.xdst[k][idx] = v;
    } else if (o.tout) {
        tg_store(o.tout + idx, v, o.tag);
    } else {
        o.fout[idx] = v;
    }
}

// NB (rows of x) and PAIR (gate/up) are compile-time so the inner loop is a
// straight run of 128-bit shared loads and FMAs with accumulators in
// registers.  One tile of a split group: segment s, accumulated into acc/acc2.
template <typename WT, int NB, bool PAIR>
__device__ __forceinline__ void gemv_tile(const GemvGeom<WT> &g, const float *__restrict__ xs, const Smem &sm, int S,
                                       uint32_t tile, int s, int nr, uint32_t *err, bool &ok, int lane, int warp,
                                       float (&acc)[sizeof(WT) == 2 ? 2 : 1][NB],
                                       float (&acc2)[sizeof(WT) == 2 ? 2 : 1][NB]) {
    constexpr int rpw = sizeof(WT) == 2 ? 2 : 1;
    const int Kp = g.Kp;
    const int st = static_cast<int>(tile % S);
    const uint32_t par = (tile / S) & 1u;
    if (ok) ok = mbar_wait(&sm.full[st], par, err, kErrTimeoutFull | 1u, g_wait_ns);
    const int c0 = s * g.kc;
    const int sw = min(g.kc, Kp - c0);
    const WT *stage = reinterpret_cast<const WT *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
    const float *xseg = xs + c0;
    if (ok && warp * rpw < nr) {
        const WT *wr = stage + static_cast<size_t>(warp * rpw) * g.kc;
#pragma unroll 2
        for (int c = lane * 4; c < sw; c += 128) {
            float4 x4[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) x4[b] = *reinterpret_cast<const float4 *>(xseg + b * Kp + c);
#pragma unroll
            for (int k = 0; k < rpw; ++k) {
                const float4 w4 = lds_w4(wr + k * g.kc + c);
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    acc[k][b] += w4.x * x4[b].x + w4.y * x4[b].y + w4.z * x4[b].z + w4.w * x4[b].w;
                if constexpr (PAIR) {
                    const float4 u4 = lds_w4(wr + (g.rps + k) * g.kc + c);
#pragma unroll
                    for (int b = 0; b < NB; ++b)
                        acc2[k][b] += u4.x * x4[b].x + u4.y * x4[b].y + u4.z * x4[b].z + u4.w * x4[b].w;
                }
            }
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
}

// Whole groups [row0, row0 + nrows) of this CTA (the same inner loop as gemv_tile, kept inline here).
template <typename WT, int NB, bool PAIR>
__device__ __forceinline__ void gemv_tiles(const GemvGeom<WT> &g, const float *__restrict__ xs, const Smem &sm, int S,
                                        uint32_t &tile, uint32_t *err, bool &ok, int tid, uint64_t *tr_first,
                                        GemvOut o) {
    constexpr int rpw = sizeof(WT) == 2 ? 2 : 1;
    const int lane = tid & 31, warp = tid >> 5;
    const int Kp = g.Kp;
    for (int grp = 0; grp < g.ngroups; ++grp) {
        const int nr = min(g.rps, g.nrows - grp * g.rps);
        float acc[rpw][NB], acc2[rpw][NB];
#pragma unroll
        for (int k = 0; k < rpw; ++k)
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[k][b] = acc2[k][b] = 0.f;
        for (int s = 0; s < g.nseg; ++s, ++tile) {
            const int st = static_cast<int>(tile % S);
            const uint32_t par = (tile / S) & 1u;
            if (ok) ok = mbar_wait(&sm.full[st], par, err, kErrTimeoutFull | 1u, g_wait_ns);
            if (grp == 0 && s == 0 && tid == 0) trace_mark(tr_first);
            const int c0 = s * g.kc;
            const int sw = min(g.kc, Kp - c0);
            const WT *stage = reinterpret_cast<const WT *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
            const float *xseg = xs + c0;
            if (ok && warp * rpw < nr) {
                const WT *wr = stage + static_cast<size_t>(warp * rpw) * g.kc;
#pragma unroll 2
                for (int c = lane * 4; c < sw; c += 128) {
                    float4 x4[NB];
#pragma unroll
                    for (int b = 0; b < NB; ++b) x4[b] = *reinterpret_cast<const float4 *>(xseg + b * Kp + c);
#pragma unroll
                    for (int k = 0; k < rpw; ++k) {
                        const float4 w4 = lds_w4(wr + k * g.kc + c);
#pragma unroll
                        for (int b = 0; b < NB; ++b)
                            acc[k][b] += w4.x * x4[b].x + w4.y * x4[b].y + w4.z * x4[b].z + w4.w * x4[b].w;
                        if constexpr (PAIR) {
                            const float4 u4 = lds_w4(wr + (g.rps + k) * g.kc + c);
#pragma unroll
                            for (int b = 0; b < NB; ++b)
                                acc2[k][b] += u4.x * x4[b].x + u4.y * x4[b].y + u4.z * x4[b].z + u4.w * x4[b].w;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[st]);
        }
#pragma unroll
        for (int k = 0; k < rpw; ++k) {
            const int j = warp * rpw + k;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float d = warp_sum(acc[k][b]);
                if constexpr (PAIR) {
                    const float u = warp_sum(acc2[k][b]);
                    if (lane == 0 && j < nr && ok) {
                        const float gelu = 0.5f * d * (1.0f + erff(d * kInvSqrt2));
                        gemv_store(o, b * o.ld + g.row0 + grp * g.rps + j, gelu * u);
                    }
                } else {
                    if (lane == 0 && j < nr && ok) gemv_store(o, b * o.ld + g.row0 + grp * g.rps + j, d);
                }
            }
        }
    }
}

// Partial row sums of a split group [kind][boundary][part][kSplitVals].
__device__ __forceinline__ float *split_slot(const DecodeParams &p, int kind, int bnd, int part) {
    return p.split_part + (static_cast<int64_t>(kind * static_cast<int>(gridDim.x) + bnd) * 2 + part) * kSplitVals;
}

// Second half of a split group's epilogue.  Each CTA has stored its partial
// sums (index (row * NB + b) * 2 + {gate, up}) in its part's slot; thread 0
// then exchanges the (forward, layer) tag into the boundary's word.  The CTA
// that finds the same tag there arrived second: it adds the two halves and
// writes the rows.  Nobody waits, so nothing can hang here; a CTA that failed
// or withholds its outputs (test hook) does not exchange, and the group's rows
// stay unwritten, as the readers' bounded waits expect.
template <int NB, bool PAIR>
static __device__ __noinline__ void gemv_split_rows(const DecodeParams &p, SmallSmem &ss, int kind, int bnd,
                                                    int layer, int64_t row0, int nr, GemvOut o, bool ok, int tid) {
    const bool all_ok = consumer_all(ok, kConsumerThreads);
    if (tid == 0) {
        uint32_t second = 0u;
        if (all_ok && !o.mute) {
            const uint64_t v = (1ull << 63) | tag_of(p, layer);
            second = atom_exch_acq_rel(p.split_tag + kind * static_cast<int>(gridDim.x) + bnd, v) == v ? 1u : 0u;
        }
        ss.split_second = second;
    }
    consumer_sync(kConsumerThreads);
    if (ss.split_second != 0u && tid < nr * NB) {
        const int j = tid / NB, b = tid - j * NB;
        const int i = (j * NB + b) * 2;
        const float *head = split_slot(p, kind, bnd, 0), *tail = split_slot(p, kind, bnd, 1);
        const float d = __ldcg(head + i) + __ldcg(tail + i);
        float v = d;
        if constexpr (PAIR) {
            const float u = __ldcg(head + i + 1) + __ldcg(tail + i + 1);
            const float gelu = 0.5f * d * (1.0f + erff(d * kInvSqrt2));
            v = gelu * u;
        }
        gemv_store(o, b * o.ld + row0 + j, v);
    }
}

// The split groups of this CTA, after its whole groups: the lead group's tail
// (part 1), then the tail group's head (part 0).  Out of line, with its
// arguments by value, so that the whole-group path around the call compiles
// as it does without it.  Returns the tile counter, and `ok` in bit 32.
template <typename WT, int NB, bool PAIR>
static __device__ __noinline__ uint64_t gemv_split_pieces(const DecodeParams &p, SmallSmem &ss, const GemvGeom<WT> g,
                                                          const float *__restrict__ xs, const Smem &sm, int S,
                                                          uint32_t tile, uint32_t *err, bool ok, int tid, GemvOut o) {
    constexpr int rpw = sizeof(WT) == 2 ? 2 : 1;
    const int lane = tid & 31, warp = tid >> 5;
    for (int k = 0; k < 2; ++k) {
        int grp, s0, s1;
        if (!g.split_piece(k, grp, s0, s1)) continue;
        const int part = k == 0 ? 1 : 0;
        const int nr = min(g.rps, g.N - grp * g.rps);
        float acc[rpw][NB], acc2[rpw][NB];
#pragma unroll
        for (int r = 0; r < rpw; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[r][b] = acc2[r][b] = 0.f;
        for (int s = s0; s < s1; ++s, ++tile) gemv_tile<WT, NB, PAIR>(g, xs, sm, S, tile, s, nr, err, ok, lane, warp, acc, acc2);
        const int bnd = part == 0 ? g.slot : g.slot - 1;
        float *mine = split_slot(p, g.kind, bnd, part);
#pragma unroll
        for (int r = 0; r < rpw; ++r) {
            const int j = warp * rpw + r;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float d = warp_sum(acc[r][b]);
                const float u = PAIR ? warp_sum(acc2[r][b]) : 0.f;
                if (lane == 0 && j < nr && ok) {
                    mine[(j * NB + b) * 2] = d;
                    mine[(j * NB + b) * 2 + 1] = u;
                }
            }
        }
        gemv_split_rows<NB, PAIR>(p, ss, g.kind, bnd, g.layer, static_cast<int64_t>(grp) * g.rps, nr, o, ok, tid);
    }
    return (static_cast<uint64_t>(ok) << 32) | tile;
}

template <typename WT, int NB>
__device__ __forceinline__ void gemv_consume(const DecodeParams &p, SmallSmem &ss, const GemvGeom<WT> &g,
                                             const float *xs, const Smem &sm, int S, uint32_t &tile, uint32_t *err,
                                             bool &ok, int tid, uint64_t *tr_first, GemvOut o) {
    if (g.pair)
        gemv_tiles<WT, NB, true>(g, xs, sm, S, tile, err, ok, tid, tr_first, o);
    else
        gemv_tiles<WT, NB, false>(g, xs, sm, S, tile, err, ok, tid, tr_first, o);
    if constexpr (sizeof(WT) == 2) {
        if (g.split) {
            const uint64_t r = g.pair ? gemv_split_pieces<WT, NB, true>(p, ss, g, xs, sm, S, tile, err, ok, tid, o)
                                      : gemv_split_pieces<WT, NB, false>(p, ss, g, xs, sm, S, tile, err, ok, tid, o);
            tile = static_cast<uint32_t>(r);
            ok = (r >> 32) != 0;
        }
    }
}

// ---------------------------------------------------------------- attention
// Split-KV attention for this CTA's items of one layer (layers.mojo:16-97):
// QK-norm + RoPE of the group's q heads and the new k, K/V write at pos,
// online-softmax over the chunk's cached positions (staged by the producer),
// partial (m, l, acc) per (row, kv head, chunk).  Returns the item count.
// HD (head dim) and GQ (q heads per kv head) are compile-time when non-zero so
// every loop unrolls and its shared/global loads issue together.
// Result of a CTA's attention items: partials written, and the consumer's
// ring position and status afterwards (returned by value so that nothing of
// the caller has to live in local memory across the call).
struct AttRet {
    uint32_t done, tile;
    bool ok;
};

template <int HD, int GQ>
__device__ __noinline__ AttRet att_items(const DecodeParams &p, const Smem &sm, SmallSmem &ss, const LayerPtrs &lp,
                                         int layer, int ph, const AttRows &a, uint32_t tile, bool ok, int tid,
                                         bool has_dep) {
    constexpr int kQ = GQ ? GQ : kMaxQPerKv;         // accumulator slots
    constexpr int kDL = HD ? HD / 32 : kMaxHeadDim / 32;  // head dims per lane
    // Head dims 64/128/256 whose q heads x dims fill whole 256-thread rounds take
    // the two-tile pass below; other shapes keep the tile-at-a-time loop.
    constexpr bool kFast = (HD == 64 || HD == 128 || HD == 256) && GQ > 0 && (GQ * HD) % kConsumerThreads == 0;
    const int G = gridDim.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int Gq = GQ ? GQ : p.Hq / p.Hkv;
    const int hd = HD ? HD : p.hd;
    const int half = hd / 2;
    const int B = p.B;
    const int hdp = HD ? HD : p.hdp;
    // shared scratch: q [Gq][hd], k, v, scores [Gq][2 * kAttTile], m/l/alpha, norm weights,
    // rope rows [B][hd], then the P.V reduction block
    float *q_s = sm.xs;
    float *k_s = q_s + Gq * hd;
    float *v_s = k_s + hd;
    float *sc = v_s + hd;
    float *m_s = sc + Gq * 2 * kAttTile;
    float *l_s = m_s + kMaxQPerKv;
    float *al_s = l_s + kMaxQPerKv;
    float *qn_s = al_s + kMaxQPerKv;
    float *kn_s = qn_s + hd;
    float *rope_s = kn_s + hd;  // [B][half cos | half sin]
    // independent of the QKV results: norm weights and this step's RoPE rows
    {
        const float *ct = lp.is_global ? p.rope_cos_g : p.rope_cos_l;
        const float *st_ = lp.is_global ? p.rope_sin_g : p.rope_sin_l;
        for (int i = tid; i < hd; i += kConsumerThreads) {
            qn_s[i] = lp.q_norm ? lp.q_norm[i] : 0.f;
            kn_s[i] = lp.k_norm ? lp.k_norm[i] : 0.f;
        }
        for (int i = tid; i < B * half; i += kConsumerThreads) {
            const int b = i / half, d = i - b * half;
            rope_s[b * hd + d] = ct[static_cast<int64_t>(ss.pos[b]) * half + d];
            rope_s[b * hd + half + d] = st_[static_cast<int64_t>(ss.pos[b]) * half + d];
        }
    }
    (void)has_dep;  // the q/k/v words are polled below
    const uint32_t tag = tag_of(p, layer);
    const float scale = p.att_scale;
    const int slot = cta_slot(ph);
    uint32_t done = 0;
    for (int item = slot; item < a.nitems; item += G) {
        int b, kvh, c, qh0;
        att_item(p, a, item, b, kvh, c, qh0);
        const int hl = qh0 - kvh * (p.Hq / p.Hkv);  // first q head within the kv group
        const int pos = ss.pos[b];
        const int t_begin = a.lo[b] + c * p.att_ch;
        const int t_end = min(t_begin + p.att_ch, pos + 1);
        // ---- raw q (Gq heads), k, v of this kv group: all loads in one round
        // trip, polled until every word carries this layer's tag
        {
            const uint64_t *qkv_b = p.qkv + static_cast<int64_t>(b) * p.qkv_rows;
            constexpr int kPer = ((GQ ? GQ : kMaxQPerKv) + 2) * (HD ? HD : kMaxHeadDim) / kConsumerThreads + 1;
            const int n = (Gq + 2) * hd;
            auto src = [&](int j) {
                const int i = tid + j * kConsumerThreads;
                const int vec = i / hd, d = i - vec * hd;
                return qkv_b + (vec < Gq ? static_cast<int64_t>(qh0 + vec) * hd + d
                                         : p.A + static_cast<int64_t>((vec == Gq ? 0 : p.Hkv) + kvh) * hd + d);
            };
            uint64_t w[kPer];
#pragma unroll
            for (int j = 0; j < kPer; ++j) w[j] = tid + j * kConsumerThreads < n ? tg_load(src(j)) : tg_pack(0.f, tag);
            ok = tg_settle(w, tag, src, p.err, 100 + ph, g_wait_ns) && ok;
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int i = tid + j * kConsumerThreads;
                if (i < n) q_s[i] = tg_val(w[j]);  // q_s, k_s, v_s are contiguous
            }
        }
        if (tid < Gq) {
            m_s[tid] = -INFINITY;
            l_s[tid] = 0.f;
        }
        consumer_sync(kConsumerThreads);
        if (tid == 0 && done == 0) trace_mark(trace_slot(p, ph, kTrAttLoaded));
        // ---- QK-norm (layers.mojo:43-49) and RoPE (52-55), one warp per vector
        for (int vec = warp; vec < Gq + 1; vec += kConsumerWarps) {
            float *x = q_s + vec * hd;
            const bool has_norm = vec < Gq ? lp.q_norm != nullptr : lp.k_norm != nullptr;
            const float *nwt = vec < Gq ? qn_s : kn_s;
            if (has_norm) {
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < kDL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hd) s += x[d] * x[d];
                }
                s = warp_sum(s);
                const float inv = rms_inv(s, p.inv_hd);
#pragma unroll
                for (int i = 0; i < kDL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hd) x[d] = x[d] * inv * (1.0f + nwt[d]);
                }
                __syncwarp();
            }
            const float *cs = rope_s + b * hd;
#pragma unroll
            for (int i0 = 0; i0 < (kDL + 1) / 2; ++i0) {
                const int i = lane + 32 * i0;
                if (i < half) {
                    const float x1 = x[i], x2 = x[i + half];
                    x[i] = x1 * cs[i] - x2 * cs[half + i];
                    x[i + half] = x2 * cs[i] + x1 * cs[half + i];
                }
            }
            __syncwarp();
        }
        consumer_sync(kConsumerThreads);
        if (tid == 0 && done == 0) trace_mark(trace_slot(p, ph, kTrAttRoped));
        // ---- K/V write at pos by the chunk that ends there (layers.mojo:57-61)
        if (t_end == pos + 1 && ss.active[b] && ok && hl == 0) {  // one item per kv head writes
            const size_t off = static_cast<size_t>(layer) * p.kv_layer_stride + static_cast<size_t>(b) * p.kv_row_stride +
                               static_cast<size_t>(kvh) * p.kv_head_stride + static_cast<size_t>(pos) * hdp;
            for (int d = tid; d < hd; d += kConsumerThreads) {
                p.kc[off + d] = k_s[d];
                p.vc[off + d] = v_s[d];
            }
        }
        if constexpr (kFast) {
            // Groups of two tiles (32 positions) at a time, one pass each:
            //  scores  thread (position sp, dim slice sl): float4 dims 4 sl + 32 j of
            //          its key row against every q head, reduced over the 8 slices
            //          with 3 shuffles;
            //  softmax one warp per head, lane = position (online across groups);
            //  P.V     thread (dims 4 dq .. 4 dq + 3, position class pq): kPPQ
            //          positions, every head; classes summed through shared memory
            //          into the running accumulators run[] (outputs tid + 256 k).
            constexpr int kGP = 2 * kAttTile;
            constexpr int kDG = HD / 4;
            constexpr int kNPQ = kConsumerThreads / kDG;
            constexpr int kPPQ = kGP / kNPQ;
            constexpr int kOut = GQ * HD / kConsumerThreads;
            float *red = rope_s + B * hd;  // [kNPQ][GQ][HD]
            float run[kOut];
#pragma unroll
            for (int k = 0; k < kOut; ++k) run[k] = 0.f;
            const int sp = tid >> 3, sl = tid & 7;
            const int dq = tid % kDG, pq = tid / kDG;
            for (int ts = t_begin; ts < t_end; ts += kGP) {
                const int np = min(kGP, t_end - ts);
                const int ntl = (np + kAttTile - 1) / kAttTile;
                const float *kt[2], *vt[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const uint32_t tu = tile + static_cast<uint32_t>(min(u, ntl - 1));
                    const int st = static_cast<int>(tu % p.S);
                    if (u < ntl && ok) ok = mbar_wait(&sm.full[st], (tu / p.S) & 1u, p.err, kErrTimeoutFull | 2u, g_wait_ns);
                    kt[u] = reinterpret_cast<const float *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
                    vt[u] = kt[u] + kAttTile * HD;
                }
                if (tid == 0 && done == 0 && ts == t_begin) trace_mark(trace_slot(p, ph, kTrPrologue));
                {
                    float acc[GQ];
#pragma unroll
                    for (int h = 0; h < GQ; ++h) acc[h] = 0.f;
                    if (sp < np) {
                        const float *kr = (ts + sp == pos) ? k_s : kt[sp >> 4] + (sp & 15) * HD;
#pragma unroll
                        for (int j = 0; j < HD / 32; ++j) {
                            const int d = 4 * sl + 32 * j;
                            const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
#pragma unroll
                            for (int h = 0; h < GQ; ++h) {
                                const float4 q4 = *reinterpret_cast<const float4 *>(q_s + h * HD + d);
                                acc[h] += q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
                            }
                        }
                    }
#pragma unroll
                    for (int h = 0; h < GQ; ++h) {
                        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
                        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
                        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 4);
                    }
                    if (sl == 0) {
#pragma unroll
                        for (int h = 0; h < GQ; ++h) sc[h * kGP + sp] = sp < np ? acc[h] * scale : -INFINITY;
                    }
                }
                consumer_sync(kConsumerThreads);
                if (warp < GQ) {  // online softmax bookkeeping (ops.mojo:139-182), lane = position
                    const int h = warp;
                    const float sv = sc[h * kGP + lane];
                    const float m_old = m_s[h];
                    const float m_new = fmaxf(m_old, warp_max(sv));
                    const float e = lane < np ? expf(sv - m_new) : 0.f;
                    sc[h * kGP + lane] = e;
                    const float es = warp_sum(e);
                    if (lane == 0) {
                        const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                        al_s[h] = alpha;
                        l_s[h] = l_s[h] * alpha + es;
                        m_s[h] = m_new;
                    }
                }
                consumer_sync(kConsumerThreads);
                {  // P @ V (layers.mojo:89-94)
                    float4 a4[GQ];
#pragma unroll
                    for (int h = 0; h < GQ; ++h) a4[h] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < kPPQ; ++i) {
                        const int pp = pq * kPPQ + i;
                        if (pp < np) {
                            const float *vr = (ts + pp == pos) ? v_s : vt[pp >> 4] + (pp & 15) * HD;
                            const float4 v4 = *reinterpret_cast<const float4 *>(vr + 4 * dq);
#pragma unroll
                            for (int h = 0; h < GQ; ++h) {
                                const float pr = sc[h * kGP + pp];
                                a4[h].x += pr * v4.x;
                                a4[h].y += pr * v4.y;
                                a4[h].z += pr * v4.z;
                                a4[h].w += pr * v4.w;
                            }
                        }
                    }
#pragma unroll
                    for (int h = 0; h < GQ; ++h) *reinterpret_cast<float4 *>(red + (pq * GQ + h) * HD + 4 * dq) = a4[h];
                }
                __syncwarp();
                if (lane == 0)
                    for (int u = 0; u < ntl; ++u) mbar_arrive(&sm.empty[(tile + u) % p.S]);
                tile += static_cast<uint32_t>(ntl);
                consumer_sync(kConsumerThreads);
#pragma unroll
                for (int k = 0; k < kOut; ++k) {
                    const int o = tid + k * kConsumerThreads;
                    const int h = o / HD, d = o - h * HD;
                    float sum = 0.f;
#pragma unroll
                    for (int q = 0; q < kNPQ; ++q) sum += red[(q * GQ + h) * HD + d];
                    run[k] = run[k] * al_s[h] + sum;
                }
                consumer_sync(kConsumerThreads);
            }
            if (tid == 0 && done == 0) trace_mark(trace_slot(p, ph, kTrAttTiles));
            // ---- partial (m, l, acc) of this chunk; combined in the o_proj prologue
            float *part = att_part(p, b, kvh, c) + hl * (hd + kPartHead);
            const int part_ld = hd + kPartHead;
#pragma unroll
            for (int k = 0; k < kOut; ++k) {
                const int o = tid + k * kConsumerThreads;
                const int h = o / HD, d = o - h * HD;
                part[h * part_ld + kPartHead + d] = run[k];
            }
            if (tid < Gq) {
                part[tid * part_ld + 0] = m_s[tid];
                part[tid * part_ld + 1] = l_s[tid];
            }
            consumer_sync(kConsumerThreads);
        } else {
        // P.V ownership: thread -> head dim pv_d, position class pv_q of ntq
        const int ntq = kConsumerThreads / hd;
        const int pv_d = tid % hd, pv_q = tid / hd;
        const bool pv_on = pv_q < ntq;
        float acc[kQ];
#pragma unroll
        for (int h = 0; h < kQ; ++h) acc[h] = 0.f;
        for (int ts = t_begin; ts < t_end; ts += kAttTile, ++tile) {
            const int st = static_cast<int>(tile % p.S);
            if (ok) ok = mbar_wait(&sm.full[st], (tile / p.S) & 1u, p.err, kErrTimeoutFull | 2u, g_wait_ns);
            if (tid == 0 && done == 0 && ts == t_begin) trace_mark(trace_slot(p, ph, kTrPrologue));
            const int nt = min(kAttTile, t_end - ts);
            const float *kt = reinterpret_cast<const float *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
            const float *vt = kt + kAttTile * hdp;
            // scores s = (q . k) * scale (layers.mojo:74-79): warp w takes positions w and w + 8,
            // lanes run over head dims, every q head accumulates at once
            {
                const int t0 = warp, t1 = warp + kConsumerWarps;
                const bool v0 = t0 < nt, v1 = t1 < nt;
                const float *k0 = (ts + t0 == pos) ? k_s : kt + t0 * hdp;
                const float *k1 = (ts + t1 == pos) ? k_s : kt + t1 * hdp;
                float s0[kQ], s1[kQ];
#pragma unroll
                for (int h = 0; h < kQ; ++h) s0[h] = s1[h] = 0.f;
#pragma unroll
                for (int i = 0; i < kDL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hd) {
                        const float ka = v0 ? k0[d] : 0.f;
                        const float kb = v1 ? k1[d] : 0.f;
#pragma unroll
                        for (int h = 0; h < kQ; ++h) {
                            if (h < Gq) {
                                const float q = q_s[h * hd + d];
                                s0[h] += q * ka;
                                s1[h] += q * kb;
                            }
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < kQ; ++h) {
                    if (h < Gq) {
                        const float a0 = warp_sum(s0[h]);
                        const float a1 = warp_sum(s1[h]);
                        if (lane == 0) {
                            if (v0) sc[h * kAttTile + t0] = a0 * scale;
                            if (v1) sc[h * kAttTile + t1] = a1 * scale;
                        }
                    }
                }
            }
            consumer_sync(kConsumerThreads);
            // online softmax bookkeeping, one warp per head
            for (int h = warp; h < Gq; h += kConsumerWarps) {
                const float s = lane < nt ? sc[h * kAttTile + lane] : -INFINITY;
                const float mx = warp_max(s);
                const float m_old = m_s[h];
                const float m_new = fmaxf(m_old, mx);
                const float e = lane < nt ? expf(s - m_new) : 0.f;
                if (lane < nt) sc[h * kAttTile + lane] = e;
                const float es = warp_sum(e);
                if (lane == 0) {
                    const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                    al_s[h] = alpha;
                    l_s[h] = l_s[h] * alpha + es;
                    m_s[h] = m_new;
                }
            }
            consumer_sync(kConsumerThreads);
            // P @ V (layers.mojo:89-94): Gq independent accumulators per thread
            if (pv_on) {
#pragma unroll
                for (int h = 0; h < kQ; ++h)
                    if (h < Gq) acc[h] *= al_s[h];
#pragma unroll 4
                for (int t = pv_q; t < nt; t += ntq) {
                    const float vv = (ts + t == pos) ? v_s[pv_d] : vt[t * hdp + pv_d];
#pragma unroll
                    for (int h = 0; h < kQ; ++h)
                        if (h < Gq) acc[h] += sc[h * kAttTile + t] * vv;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[st]);
            consumer_sync(kConsumerThreads);
        }
        if (tid == 0 && done == 0) trace_mark(trace_slot(p, ph, kTrAttTiles));
        // ---- partial (m, l, acc) of this chunk; combined in the o_proj prologue
        float *part = att_part(p, b, kvh, c) + hl * (hd + kPartHead);
        const int part_ld = hd + kPartHead;
        if (ntq > 1) {  // fold the position classes
            float *red = rope_s + B * hd;  // [ntq][Gq][hd]
            if (pv_on)
#pragma unroll
                for (int h = 0; h < kQ; ++h)
                    if (h < Gq) red[(pv_q * Gq + h) * hd + pv_d] = acc[h];
            consumer_sync(kConsumerThreads);
            if (pv_q == 0) {
#pragma unroll
                for (int h = 0; h < kQ; ++h) {
                    if (h < Gq) {
                        float s = 0.f;
                        for (int q = 0; q < ntq; ++q) s += red[(q * Gq + h) * hd + pv_d];
                        acc[h] = s;
                    }
                }
            }
        }
        if (pv_q == 0) {
#pragma unroll
            for (int h = 0; h < kQ; ++h)
                if (h < Gq) part[h * part_ld + kPartHead + pv_d] = acc[h];
        }
        if (tid < Gq) {
            part[tid * part_ld + 0] = m_s[tid];
            part[tid * part_ld + 1] = l_s[tid];
        }
        consumer_sync(kConsumerThreads);
        }
        if (tid == 0 && done == 0) trace_mark(trace_slot(p, ph, kTrAttPart));
        ++done;
    }
    return AttRet{done, tile, ok};
}

__device__ __forceinline__ AttRet att_dispatch(const DecodeParams &p, const Smem &sm, SmallSmem &ss,
                                               const LayerPtrs &lp, int layer, int ph, const AttRows &a,
                                               uint32_t tile, bool ok, int tid, bool has_dep) {
    const int Gq = p.Hq / p.Hkv;
    if (p.att_split && p.hd == 256) return att_items<256, 1>(p, sm, ss, lp, layer, ph, a, tile, ok, tid, has_dep);
#define MG_ATT(HD_, GQ_) \
    if (p.hd == HD_ && Gq == GQ_) return att_items<HD_, GQ_>(p, sm, ss, lp, layer, ph, a, tile, ok, tid, has_dep);
    MG_ATT(256, 4)
    MG_ATT(256, 3)
    MG_ATT(256, 2)
    MG_ATT(256, 1)
    MG_ATT(128, 2)
    MG_ATT(128, 4)
    MG_ATT(64, 4)
#undef MG_ATT
    return att_items<0, 0>(p, sm, ss, lp, layer, ph, a, tile, ok, tid, has_dep);
}

// o_proj input from the split-KV partials of every (row, kv head):
//   w_c = exp(m_c - M) / sum_c l_c exp(m_c - M);  x[b][h*hd+d] = sum_c w_c * acc_c[d]
// One warp per (row, q head, half of the head dims): lane c holds chunk c's
// m and l, and every chunk's 4-dim slice of acc is loaded as a float4 in the
// same round trip (16 chunks per batch).  Head dims that are not a multiple
// of 4 take the scalar path.
static __device__ __noinline__ void att_combine(const DecodeParams &p, const AttRows &a, int Kp, float *xs, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int Gq = p.Hq / p.Hkv, hd = p.hd, B = p.B;
    const int part_ld = hd + kPartHead;
    const int64_t cstride = static_cast<int64_t>(Gq) * part_ld;
    if (hd % 4 == 0) {
        constexpr int kBatch = 16;
        const int halves = hd > 128 ? 2 : 1;
        const int dpt = hd / halves;  // dims per task, <= 128: one float4 per lane
        for (int task = warp; task < B * p.Hq * halves; task += kConsumerWarps) {
            const int bh = task / halves, hf = task - bh * halves;
            const int b = bh / p.Hq, hq = bh - b * p.Hq;
            const int kvh = hq / Gq, hl = hq - kvh * Gq;
            const int nch = a.nch[b];
            const float *base = att_part(p, b, kvh, 0) + hl * part_ld;
            const int d0 = hf * dpt + lane * 4;
            const bool on = lane * 4 < dpt;
            float m = -INFINITY, l = 0.f;
            if (lane < nch) {
                m = __ldcg(base + lane * cstride);
                l = __ldcg(base + lane * cstride + 1);
            }
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            float w = 0.f;
            for (int c0 = 0; c0 < nch; c0 += kBatch) {
                float4 v[kBatch];
#pragma unroll
                for (int u = 0; u < kBatch; ++u)
                    v[u] = (on && c0 + u < nch)
                               ? __ldcg(reinterpret_cast<const float4 *>(base + (c0 + u) * cstride + kPartHead + d0))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
                if (c0 == 0) {
                    const float M = warp_max(m);
                    const float e = lane < nch ? expf(m - M) : 0.f;
                    w = __fdividef(e, warp_sum(l * e));
                }
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    const float wu = __shfl_sync(0xffffffffu, w, (c0 + u) & 31);
                    x.x += wu * v[u].x;
                    x.y += wu * v[u].y;
                    x.z += wu * v[u].z;
                    x.w += wu * v[u].w;
                }
            }
            if (on) *reinterpret_cast<float4 *>(xs + b * Kp + hq * hd + d0) = x;
        }
    } else {
        constexpr int kDims = kMaxHeadDim / 32;
        constexpr int kCh = 8;
        for (int bh = warp; bh < B * p.Hq; bh += kConsumerWarps) {
            const int b = bh / p.Hq, hq = bh - b * p.Hq;
            const int kvh = hq / Gq, hl = hq - kvh * Gq;
            const int nch = a.nch[b];
            const float *base = att_part(p, b, kvh, 0) + hl * part_ld;
            float m = -INFINITY, l = 0.f;
            if (lane < nch) {
                m = __ldcg(base + lane * cstride);
                l = __ldcg(base + lane * cstride + 1);
            }
            const float M = warp_max(m);
            const float e = lane < nch ? expf(m - M) : 0.f;
            const float w = __fdividef(e, warp_sum(l * e));
            float x[kDims];
#pragma unroll
            for (int i = 0; i < kDims; ++i) x[i] = 0.f;
            for (int c0 = 0; c0 < nch; c0 += kCh) {
                float v[kCh][kDims];
#pragma unroll
                for (int u = 0; u < kCh; ++u)
#pragma unroll
                    for (int i = 0; i < kDims; ++i) {
                        const int d = lane + 32 * i;
                        v[u][i] = (c0 + u < nch && d < hd) ? __ldcg(base + (c0 + u) * cstride + kPartHead + d) : 0.f;
                    }
#pragma unroll
                for (int u = 0; u < kCh; ++u) {
                    const float wu = __shfl_sync(0xffffffffu, w, (c0 + u) & 31);
#pragma unroll
                    for (int i = 0; i < kDims; ++i) x[i] += wu * v[u][i];
                }
            }
#pragma unroll
            for (int i = 0; i < kDims; ++i) {
                const int d = lane + 32 * i;
                if (d < hd) xs[b * Kp + hq * hd + d] = x[i];
            }
        }
    }
    for (int o = tid; o < B * Kp; o += kConsumerThreads) {
        const int b = o / Kp, oo = o - b * Kp;
        if (oo >= p.A) xs[b * Kp + oo] = 0.f;
    }
    consumer_sync(kConsumerThreads);
}

// Per-CTA top-k of the lm_head rows (keys to cand_key).  The CTA's logits are
// staged in the (now idle) ring first: one batched read instead of a round
// trip per radix pass.
static __device__ __noinline__ void lm_topk(const DecodeParams &p, const Smem &sm, int64_t row0, int nrows, int tid) {
    const int G = gridDim.x;
    SelectSmem &sel = *reinterpret_cast<SelectSmem *>(sm.xs);
    uint64_t *outk = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(sm.xs) + sizeof(SelectSmem));
    float *lg = reinterpret_cast<float *>(sm.ring);  // nrows <= V / G + 1 floats, far below one stage
    for (int b = 0; b < p.B; ++b) {
        const float *lr = p.logits + static_cast<int64_t>(b) * p.V + row0;
        for (int i0 = 0; i0 < nrows; i0 += 8 * kConsumerThreads) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + tid + j * kConsumerThreads;
                v[j] = i < nrows ? lr[i] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + tid + j * kConsumerThreads;
                if (i < nrows) lg[i] = v[j];
            }
        }
        consumer_sync(kConsumerThreads);
        const uint32_t r0 = static_cast<uint32_t>(row0 + p.vocab_off);  // global token ids
        block_select_topk(
            nrows, p.topk, [&](int i) { return topk_key(lg[i], r0 + static_cast<uint32_t>(i)); }, outk, sel, tid,
            kConsumerThreads, [] { consumer_sync(kConsumerThreads); });
        if (p.tp > 1) {  // to every rank's candidate block [tp][xB][G][kMaxTopK], slot of this rank
            const int64_t off = ((static_cast<int64_t>(p.tp_rank) * p.xB + b) * G + blockIdx.x) * kMaxTopK;
            for (int r = 0; r < p.tp; ++r) {
                uint64_t *dst = reinterpret_cast<uint64_t *>(p.xpeer[r] + p.x_cand) + off;
                for (int j = tid; j < p.topk; j += kConsumerThreads) dst[j] = outk[j];
            }
        } else {
            uint64_t *dst = p.cand_key + (static_cast<int64_t>(b) * G + blockIdx.x) * kMaxTopK;
            for (int j = tid; j < p.topk; j += kConsumerThreads) dst[j] = outk[j];
        }
        consumer_sync(kConsumerThreads);
    }
}

// Merge of all CTAs' candidates for row b and the draw (model.py:103-150).
// Every CTA's list holds its K best keys, sorted.  For K > kHead the K best
// of all lists are first looked for among the heads (first kHead keys) of the
// lists: they are the true K best whenever the K-th of them beats every list's
// next key (key kHead), which holds unless one list holds more than kHead of
// the winners; otherwise all keys are merged.  Keys are staged in the idle ring.
static __device__ __noinline__ int32_t row_draw(const DecodeParams &p, const Smem &sm, int b, bool ok, int tid) {
    constexpr int kHead = 8;
    const int G = gridDim.x;
    SelectSmem &sel = *reinterpret_cast<SelectSmem *>(sm.xs);
    unsigned char *after = reinterpret_cast<unsigned char *>(sm.xs) + sizeof(SelectSmem);
    uint64_t *outk = reinterpret_cast<uint64_t *>(after);
    double *fscr = reinterpret_cast<double *>(after + kMaxTopK * sizeof(uint64_t));
    double *escr = fscr + kMaxTopK;
    int *oscr = reinterpret_cast<int *>(escr + kMaxTopK);
    int *ish = oscr + kMaxTopK;  // [4]
    // candidates (rank s, CTA g, k): tp = 1 reads this rank's cand_key; tp > 1
    // the exchange block that every rank wrote its CTAs' candidates into
    const uint64_t *ck = p.tp > 1 ? reinterpret_cast<const uint64_t *>(p.xpeer[p.tp_rank] + p.x_cand) +
                                        static_cast<int64_t>(b) * G * kMaxTopK
                                  : p.cand_key + static_cast<int64_t>(b) * G * kMaxTopK;
    const int64_t sstride = static_cast<int64_t>(p.xB) * G * kMaxTopK;
    const int K = p.topk;
    const int nl = p.tp * G;  // lists
    auto list = [&](int l) {
        const int s = l / G, g = l - s * G;
        return ck + s * sstride + static_cast<int64_t>(g) * kMaxTopK;
    };
    auto sync = [] { consumer_sync(kConsumerThreads); };
    uint64_t *keys = reinterpret_cast<uint64_t *>(sm.ring);
    bool merged = false;
    if (K > kHead && static_cast<size_t>(nl) * (kHead + 1) * sizeof(uint64_t) <= static_cast<size_t>(p.S) * kStageBytes) {
        uint64_t *nxt = keys + nl * kHead;  // key kHead of every list
        const int tot = nl * (kHead + 1);
        for (int i0 = 0; i0 < tot; i0 += 8 * kConsumerThreads) {
            uint64_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + tid + j * kConsumerThreads;
                v[j] = i < tot ? __ldcg(list(i / (kHead + 1)) + i % (kHead + 1)) : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + tid + j * kConsumerThreads;
                if (i < tot) {
                    const int l = i / (kHead + 1), k = i - l * (kHead + 1);
                    if (k < kHead) keys[l * kHead + k] = v[j];
                    else nxt[l] = v[j];
                }
            }
        }
        sync();
        block_select_topk(nl * kHead, K, [&](int i) { return keys[i]; }, outk, sel, tid, kConsumerThreads, sync);
        uint64_t m = 0;
        for (int l = tid; l < nl; l += kConsumerThreads) m = nxt[l] > m ? nxt[l] : m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t other = __shfl_xor_sync(0xffffffffu, m, o);
            m = other > m ? other : m;
        }
        if ((tid & 31) == 0) sel.tmp[tid >> 5] = m;
        sync();
        if (tid == 0) {
            uint64_t mx = 0;
            for (int w = 0; w < kConsumerWarps; ++w) mx = sel.tmp[w] > mx ? sel.tmp[w] : mx;
            ish[0] = outk[K - 1] > mx ? 1 : 0;
        }
        sync();
        merged = ish[0] != 0;
        sync();
    }
    if (!merged) {
        const int GK = G * K;
        const int n = p.tp * GK;
        auto cand_at = [&](int i) {
            const int s = i / GK, r = i - s * GK;
            return __ldcg(ck + s * sstride + (r / K) * kMaxTopK + (r % K));
        };
        if (static_cast<size_t>(n) * sizeof(uint64_t) > static_cast<size_t>(p.S) * kStageBytes) {  // ring too small
            block_select_topk(n, K, cand_at, outk, sel, tid, kConsumerThreads, sync);
        } else {
            for (int i0 = 0; i0 < n; i0 += 16 * kConsumerThreads) {
                uint64_t v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int i = i0 + tid + j * kConsumerThreads;
                    v[j] = i < n ? cand_at(i) : 0ull;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int i = i0 + tid + j * kConsumerThreads;
                    if (i < n) keys[i] = v[j];
                }
            }
            sync();
            block_select_topk(n, K, [&](int i) { return keys[i]; }, outk, sel, tid, kConsumerThreads, sync);
        }
    }
    const double u = p.uniforms ? p.uniforms[b] : philox_uniform(p.seed, p.rng_offset, b + p.row_base);
    const int32_t token = draw_block(outk, K, p.temperature, p.top_p, u, fscr, escr, oscr, ish, tid, kConsumerThreads,
                                     sync);
    return (tid == 0 && ok) ? token : -1;
}

// ---------------------------------------------------------------- consumer phases
template <typename WT, int NB, bool TP>
__device__ void consumer_run(const DecodeParams &p, const Smem &sm, SmallSmem &ss, int tid) {
    const int G = gridDim.x;
    constexpr int B = NB;
    bool ok = ld_relaxed_u32(p.err) == 0u;
    uint32_t tile = 0;
    for (int ph = p.ph_begin; ph < p.ph_end; ++ph) {
        int kind, layer;
        phase_of(ph, p.L, kind, layer);
        const LayerPtrs &lp = sm.layers[layer];
        const bool has_dep = ph - 1 >= p.ph_begin;
        // test hook: one CTA with work in this phase withholds its outputs (the last
        // slot always owns rows of a projection; slot 0 owns attention item 0)
        const bool mute = ph == p.stall_phase && cta_slot(ph) == (kind == PH_ATT ? 0 : G - 1);
        auto muted = [mute](GemvOut o) {
            o.mute = mute;
            return o;
        };
        if (tid == 0) {
            trace_mark(trace_slot(p, ph, kTrStart));
            ss.tr_ready = trace_slot(p, ph, kTrReady);
            ss.tr_end = trace_slot(p, ph, kTrEnd);
        }
        if (kind == PH_QKV) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            const uint32_t tag = tag_of(p, layer);
            uint64_t *out_h = (blockIdx.x == 0) ? p.h : nullptr;
            if (layer == 0) {
                stage_embed<WT, NB>(static_cast<const WT *>(p.embed), p.embed_ld, ss.tok, lp.in_ln, out_h, tag, p.H,
                                    p.inv_h, p.emb_scale, g.Kp, sm.xs, ss, tid);
            } else {
                const LayerPtrs &prev = sm.layers[layer - 1];
                NormW nw;
                norm_prefetch(nw, prev.post_ff_ln, lp.in_ln, p.H, tid);
                // x = r + norm(mlp, post_ff) (layers.mojo:216-220), xs = norm(x, input_layernorm) (195)
                if constexpr (TP) {  // mlp = the sum of every rank's down_proj partial of layer - 1
                    ok = xwait(p, 1, p.xep + layer - 1, 100 + ph, ss, tid) && ok;
                    ok = stage_norm<NB, true>(p.r, nullptr, xrecv(p, p.tp_rank, 1), tag - 1, prev.post_ff_ln,
                                              lp.in_ln, nw, out_h, tag, p.H, p.inv_h, g.Kp, sm.xs, ss, tid, p.err,
                                              100 + ph, p.tp, static_cast<int64_t>(p.xB) * p.H) && ok;
                } else {
                    ok = stage_norm<NB>(p.r, p.mlp_raw, nullptr, tag - 1, prev.post_ff_ln, lp.in_ln, nw, out_h, tag,
                                        p.H, p.inv_h, g.Kp, sm.xs, ss, tid, p.err, 100 + ph) && ok;
                }
            }
            if (tid == 0) trace_mark(ss.tr_ready);
            gemv_consume<WT, NB>(p, ss, g, sm.xs, sm, p.S, tile, p.err, ok, tid, trace_slot(p, ph, kTrPrologue),
                                 muted(gemv_out_tagged(p.qkv, p.qkv_rows, tag)));
            phase_done(ss, tid);
        } else if (kind == PH_ATT) {
            if (tid == 0) att_rows<NB>(p, lp.is_global != 0, ss.pos, ss.att);
            consumer_sync(kConsumerThreads);
            const AttRet r = att_dispatch(p, sm, ss, lp, layer, ph, ss.att, tile, ok, tid, has_dep);
            tile = r.tile;
            ok = r.ok;
            cta_signal(ctr_phase(p, ph), mute ? 0u : r.done, ss, tid);
        } else if (kind == PH_O) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            const uint32_t tag = tag_of(p, layer);
            if (tid == 0) att_rows<NB>(p, lp.is_global != 0, ss.pos, ss.att);
            consumer_sync(kConsumerThreads);
            if (has_dep)
                ok = cta_wait(ctr_phase(p, ph - 1), static_cast<uint32_t>(ss.att.nitems), p.err, 100 + ph, ss, tid) &&
                     ok;
            att_combine(p, ss.att, g.Kp, sm.xs, tid);
            // with tensor parallelism the row-split o_proj partials go to every rank
            gemv_consume<WT, NB>(p, ss, g, sm.xs, sm, p.S, tile, p.err, ok, tid, trace_slot(p, ph, kTrPrologue),
                                 muted(TP ? gemv_out_peers(ss.xdst_o, p.tp, p.H) : gemv_out_tagged(p.o_raw, p.H, tag)));
            phase_done(ss, tid);
            if constexpr (TP) xsignal(p, 0, tid);
        } else if (kind == PH_GU) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            const uint32_t tag = tag_of(p, layer);
            NormW nw;
            norm_prefetch(nw, lp.post_attn_ln, lp.pre_ff_ln, p.H, tid);
            uint64_t *out_r = blockIdx.x == 0 ? p.r : nullptr;
            // r = h + norm(o_raw, post_attn) (layers.mojo:202-207); xs = norm(r, pre_ff) (209-210)
            if constexpr (TP) {  // o_raw = the sum of every rank's o_proj partial
                ok = xwait(p, 0, p.xep + layer, 100 + ph, ss, tid) && ok;
                ok = stage_norm<NB, true>(p.h, nullptr, xrecv(p, p.tp_rank, 0), tag, lp.post_attn_ln, lp.pre_ff_ln,
                                          nw, out_r, tag, p.H, p.inv_h, g.Kp, sm.xs, ss, tid, p.err, 100 + ph, p.tp,
                                          static_cast<int64_t>(p.xB) * p.H) && ok;
            } else {
                ok = stage_norm<NB>(p.h, p.o_raw, nullptr, tag, lp.post_attn_ln, lp.pre_ff_ln, nw, out_r, tag, p.H,
                                    p.inv_h, g.Kp, sm.xs, ss, tid, p.err, 100 + ph) && ok;
            }
            if (tid == 0) trace_mark(ss.tr_ready);
            gemv_consume<WT, NB>(p, ss, g, sm.xs, sm, p.S, tile, p.err, ok, tid, trace_slot(p, ph, kTrPrologue),
                                 muted(gemv_out_float(p.act, p.Ip)));
            cta_signal(ctr_phase(p, ph), mute ? 0u : 1u, ss, tid);
        } else if (kind == PH_D) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            const uint32_t tag = tag_of(p, layer);
            if (has_dep) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
            // down_proj input: act rows, 8 float4 loads in flight per thread
            for (int b = 0; b < B; ++b) {
                for (int i0 = 0; i0 < g.Kp; i0 += 8 * 4 * kConsumerThreads) {
                    float4 v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int i = i0 + (tid + j * kConsumerThreads) * 4;
                        v[j] = i < g.Kp ? __ldcg(reinterpret_cast<const float4 *>(p.act + static_cast<int64_t>(b) * p.Ip + i))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int i = i0 + (tid + j * kConsumerThreads) * 4;
                        if (i < g.Kp) *reinterpret_cast<float4 *>(sm.xs + b * g.Kp + i) = v[j];
                    }
                }
            }
            consumer_sync(kConsumerThreads);
            gemv_consume<WT, NB>(p, ss, g, sm.xs, sm, p.S, tile, p.err, ok, tid, trace_slot(p, ph, kTrPrologue),
                                 muted(TP ? gemv_out_peers(ss.xdst_d, p.tp, p.H) : gemv_out_tagged(p.mlp_raw, p.H, tag)));
            phase_done(ss, tid);
            if constexpr (TP) xsignal(p, 1, tid);
        } else if (kind == PH_LMH) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            if (p.lm_mode != kLmNone) {
                NormW nw;
                norm_prefetch(nw, lp.post_ff_ln, p.final_norm, p.H, tid);
                // x = r + norm(mlp_raw, post_ff); xs = norm(x, final norm) (layers.mojo:283-285)
                const uint32_t tag = tag_of(p, p.L - 1);
                if constexpr (TP) {
                    ok = xwait(p, 1, p.xep + p.L - 1, 100 + ph, ss, tid) && ok;
                    ok = stage_norm<NB, true>(p.r, nullptr, xrecv(p, p.tp_rank, 1), tag, lp.post_ff_ln, p.final_norm,
                                              nw, nullptr, 0u, p.H, p.inv_h, g.Kp, sm.xs, ss, tid, p.err, 100 + ph,
                                              p.tp, static_cast<int64_t>(p.xB) * p.H) && ok;
                } else {
                    ok = stage_norm<NB>(p.r, p.mlp_raw, nullptr, tag, lp.post_ff_ln, p.final_norm, nw, nullptr, 0u,
                                        p.H, p.inv_h, g.Kp, sm.xs, ss, tid, p.err, 100 + ph) && ok;
                }
            }
            if (p.lm_mode == kLmEmbed) {
                if (blockIdx.x == 0 && ok)
                    for (int b = 0; b < B; ++b)
                        if (ss.active[b])
                            for (int i = tid; i < p.H; i += kConsumerThreads)
                                p.emb_acc[static_cast<int64_t>(b) * p.H + i] += sm.xs[b * g.Kp + i];
            } else if (p.lm_mode == kLmLogits) {
                gemv_consume<WT, NB>(p, ss, g, sm.xs, sm, p.S, tile, p.err, ok, tid, trace_slot(p, ph, kTrPrologue),
                                     muted(gemv_out_float(p.logits, p.V)));
                if (p.topk > 0) {
                    consumer_sync(kConsumerThreads);
                    lm_topk(p, sm, g.row0, g.nrows, tid);
                }
            }
            cta_signal(ctr_phase(p, ph), mute ? 0u : 1u, ss, tid);
            // every rank's logits and candidates are complete once this exchange is counted
            if constexpr (TP)
                if (p.lm_mode == kLmLogits) xsignal(p, 2, tid);
        } else {  // PH_SAMPLE
            const int b = blockIdx.x;
            if (b < B) {
                int32_t token = -1;
                if constexpr (TP) {
                    if (p.lm_mode == kLmLogits) ok = xwait(p, 2, p.lm_ep, 100 + ph, ss, tid) && ok;
                    if (p.sample && p.lm_mode == kLmLogits && p.topk > 0) token = row_draw(p, sm, b, ok, tid);
                } else if (p.sample && p.lm_mode == kLmLogits && p.topk > 0) {
                    if (has_dep) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                    token = row_draw(p, sm, b, ok, tid);
                }
                if (tid == 0 && ok) {
                    if (token >= 0) {
                        p.tok[b] = token;
                        if (p.out_tokens) p.out_tokens[b] = token;
                    }
                    if (ss.active[b]) p.pos[b] = ss.pos[b] + 1;
                }
            }
        }
    }
}

// ---------------------------------------------------------------- producer
template <typename WT, int NB>
__device__ void producer_run(const DecodeParams &p, const Smem &sm, SmallSmem &ss) {
    const int G = gridDim.x;
    const uint64_t pol_w = policy_evict_first();
    uint32_t tile = 0, issued = 0;
    bool ok = true;
    const uint32_t S = static_cast<uint32_t>(p.S);
    const uint32_t inflight = static_cast<uint32_t>(min(max(p.max_inflight, 1), p.S));
    // Slot for tile t: its stage was released by the consumers (tile t - S), and
    // at most `inflight` copies are outstanding (tile t - inflight has landed).
    auto acquire_slot = [&](uint32_t t) -> bool {
        if (t >= S && !mbar_wait(&sm.empty[t % S], ((t / S) - 1) & 1u, p.err, kErrTimeoutEmpty | 1u, g_wait_ns)) return false;
        if (t >= inflight) {
            const uint32_t u = t - inflight;
            if (u < issued && !mbar_wait(&sm.full[u % S], (u / S) & 1u, p.err, kErrTimeoutFull | 3u, g_wait_ns)) return false;
        }
        return true;
    };
    for (int ph = p.ph_begin; ph < p.ph_end; ++ph) {
        int kind, layer;
        phase_of(ph, p.L, kind, layer);
        const LayerPtrs &lp = sm.layers[layer];
        trace_mark(trace_slot(p, ph, kTrProdStart));
        if (kind == PH_ATT) {
            AttRows &a = ss.att_p;
            att_rows<NB>(p, lp.is_global != 0, ss.pos, a);
            const int slot = cta_slot(ph);
            for (int item = slot; item < a.nitems; item += G) {
                int b, kvh, c, qh0;
                att_item(p, a, item, b, kvh, c, qh0);
                const int pos = ss.pos[b];
                const int t_begin = a.lo[b] + c * p.att_ch;
                const int t_end = min(t_begin + p.att_ch, pos + 1);
                const size_t kvbase = static_cast<size_t>(layer) * p.kv_layer_stride +
                                      static_cast<size_t>(b) * p.kv_row_stride +
                                      static_cast<size_t>(kvh) * p.kv_head_stride;
                for (int ts = t_begin; ts < t_end; ts += kAttTile, ++tile) {
                    const int st = static_cast<int>(tile % S);
                    ok = ok && acquire_slot(tile);
                    const int te = min(ts + kAttTile, t_end);
                    const int ncached = max(0, min(te, pos) - ts);  // row `pos` is computed, not read
                    const uint32_t bytes = static_cast<uint32_t>(ncached * p.hdp * 4);
                    if (!ok) continue;
                    issued = tile + 1;
                    mbar_arrive_expect_tx(&sm.full[st], 2u * bytes);
                    if (bytes) {
                        unsigned char *dst = sm.ring + static_cast<size_t>(st) * kStageBytes;
                        const size_t off = kvbase + static_cast<size_t>(ts) * p.hdp;
                        bulk_g2s(dst, p.kc + off, bytes, &sm.full[st], pol_w);
                        bulk_g2s(dst + static_cast<size_t>(kAttTile) * p.hdp * 4, p.vc + off, bytes, &sm.full[st],
                                 pol_w);
                    }
                }
            }
        } else if (kind != PH_SAMPLE) {
            GemvGeom<WT> g;
            gemv_geom<WT>(p, lp, kind, ph, g);
            // this CTA's tiles are contiguous in the tiled layout: one bulk copy per tile
            const uint32_t bytes = static_cast<uint32_t>(g.tile_elems * sizeof(WT));
            const int ntiles = g.ngroups * g.nseg;
            if (p.pf_tiles > 0 && ok && !g.split && ntiles > static_cast<int>(S)) {
                // L2 prefetch of the part of this phase the ring cannot hold yet
                const char *from = reinterpret_cast<const char *>(g.tiles) + static_cast<size_t>(S) * bytes;
                size_t left = static_cast<size_t>(ntiles - static_cast<int>(S)) * bytes;
                for (; left > 0;) {
                    const uint32_t nb = static_cast<uint32_t>(min(left, static_cast<size_t>(1u << 20)));
                    bulk_prefetch_l2(from, nb);
                    from += nb;
                    left -= nb;
                }
            }
            for (int t = 0; t < ntiles; ++t, ++tile) {
                const int st = static_cast<int>(tile % S);
                ok = ok && acquire_slot(tile);
                if (!ok) continue;
                issued = tile + 1;
                mbar_arrive_expect_tx(&sm.full[st], bytes);
                bulk_g2s(sm.ring + static_cast<size_t>(st) * kStageBytes, g.tiles + static_cast<int64_t>(t) * g.tile_elems,
                         bytes, &sm.full[st], pol_w);
            }
            // then the split groups' parts, in the consumers' order (gemv_split_pieces)
            for (int k = 0; sizeof(WT) == 2 && g.split && k < 2; ++k) {
                int grp, s0, s1;
                if (!g.split_piece(k, grp, s0, s1)) continue;
                for (int sg = s0; sg < s1; ++sg, ++tile) {
                    const int st = static_cast<int>(tile % S);
                    ok = ok && acquire_slot(tile);
                    if (!ok) continue;
                    issued = tile + 1;
                    mbar_arrive_expect_tx(&sm.full[st], bytes);
                    bulk_g2s(sm.ring + static_cast<size_t>(st) * kStageBytes,
                             g.base + (static_cast<int64_t>(grp) * g.nseg + sg) * g.tile_elems, bytes, &sm.full[st],
                             pol_w);
                }
            }
        }
        trace_mark(trace_slot(p, ph, kTrProdEnd));
    }
    // Drain: copies still in flight must land before the CTA exits.
    const uint32_t first = issued > S ? issued - S : 0u;
    for (uint32_t t = first; t < issued; ++t) {
        if (!mbar_wait_drain(&sm.full[t % S], (t / S) & 1u)) set_error(p.err, kErrTimeoutDrain);
    }
}

// ---------------------------------------------------------------- the kernel
template <typename WT, int NB, bool TP>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ SmallSmem ss;
    // The pointer block lives in shared memory: helpers take it by reference,
    // and a local copy would turn each of their reads into a local-memory load.
    __shared__ Smem sm;
    Smem sl;
    {
        uintptr_t base = reinterpret_cast<uintptr_t>(smem_raw);
        base = (base + 127) & ~static_cast<uintptr_t>(127);
        sl.ring = reinterpret_cast<unsigned char *>(base);
        sl.xs = reinterpret_cast<float *>(sl.ring + static_cast<size_t>(p.S) * kStageBytes);
        sl.full = reinterpret_cast<uint64_t *>(sl.xs + p.xs_floats);
        sl.empty = sl.full + p.S;
        sl.layers = reinterpret_cast<LayerPtrs *>(sl.empty + p.S);
    }
    if (threadIdx.x == 0) {
        sm = sl;
        g_wait_ns = p.wait_ns ? p.wait_ns : kWaitBudgetNs;
    }
    const int tid = threadIdx.x;
    const int G = gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < p.S; ++s) {
            mbar_init(&sl.full[s], 1);
            mbar_init(&sl.empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(p.layers);
        uint32_t *dst = reinterpret_cast<uint32_t *>(sl.layers);
        const int nw = p.L * static_cast<int>(sizeof(LayerPtrs) / 4);
        for (int i = tid; i < nw; i += kThreads) dst[i] = src[i];
    }
    if (tid < p.B) {
        const int b = tid;
        int active = 1;
        int tok;
        if (p.ids != nullptr) {
            const int nv = p.nvalid[b];
            active = p.step_t < nv;
            const int ti = min(p.step_t, max(nv - 1, 0));
            tok = p.ids[static_cast<int64_t>(b) * p.ids_ld + ti];
        } else {
            tok = p.tok[b];
        }
        if (tok < 0 || tok >= p.V_full) {
            set_error(p.err, kErrBadToken | static_cast<uint32_t>(b));
            tok = 0;
        }
        int pos = p.pos[b];
        if (pos < 0 || pos >= p.cap) {
            if (active) set_error(p.err, kErrBadPos | static_cast<uint32_t>(b));
            active = 0;
            pos = min(max(pos, 0), p.cap - 1);
        }
        ss.pos[b] = pos;
        ss.tok[b] = tok;
        ss.active[b] = active;
    }
    if (TP && tid == 0) {  // this rank's receive block on every rank
        for (int r = 0; r < p.tp; ++r) {
            const int64_t blk = static_cast<int64_t>(p.tp_rank) * p.xB * p.H;
            ss.xdst_o[r] = xrecv(p, r, 0) + blk;
            ss.xdst_d[r] = xrecv(p, r, 1) + blk;
        }
    }
    __syncthreads();
    uint64_t *tr_kernel =
        p.trace ? p.trace + static_cast<size_t>(G) * p.n_phases * kTraceSlots + 2 * blockIdx.x : nullptr;
    if (tid == 0) {
        trace_mark(tr_kernel);
        // SM clock cross-check for the timeline: cycles at kernel begin in the SAMPLE phase's spare slot
        uint64_t *ck = trace_slot(p, p.n_phases - 1, 6);
        if (ck) *ck = clock64();
    }

    if ((tid >> 5) == kConsumerWarps) {
        if ((tid & 31) == 0) producer_run<WT, NB>(p, sm, ss);
    } else {
        consumer_run<WT, NB, TP>(p, sm, ss, tid);
    }

    // ---- exit: the last CTA out resets the counters used by this launch.
    __syncthreads();
    if (tid == 0) {
        trace_mark(tr_kernel ? tr_kernel + 1 : nullptr);
        uint64_t *ck = trace_slot(p, p.n_phases - 1, 7);
        if (ck) *ck = clock64();
        __threadfence();
        const uint32_t old = atomicAdd(ctr_exit(p), 1u);
        if (old == static_cast<uint32_t>(G - 1)) {
            __threadfence();
            for (int ph = p.ph_begin; ph < p.ph_end; ++ph) *ctr_phase(p, ph) = 0u;
            *ctr_exit(p) = 0u;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------- host launch (per row count)
// Static shared memory of the kernel (SmallSmem and the pointer block) in bytes.
template <typename WT, int NB>
size_t decode_static_smem_nb() {
    size_t m = 0;
    cudaFuncAttributes a;
    if (cudaFuncGetAttributes(&a, decode_kernel<WT, NB, false>) != cudaSuccess) return 2048;
    m = a.sharedSizeBytes;
    if (cudaFuncGetAttributes(&a, decode_kernel<WT, NB, true>) != cudaSuccess) return 2048;
    return m > a.sharedSizeBytes ? m : a.sharedSizeBytes;
}

template <typename WT, int NB>
cudaError_t decode_prepare_nb(size_t dynamic_smem) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<WT, NB, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(dynamic_smem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(decode_kernel<WT, NB, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(dynamic_smem));
}

template <typename WT, int NB>
int decode_occupancy_nb(size_t smem) {
    int n0 = 0, n1 = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n0, decode_kernel<WT, NB, false>, kThreads, smem) !=
        cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n1, decode_kernel<WT, NB, true>, kThreads, smem) !=
        cudaSuccess)
        return 0;
    return n0 < n1 ? n0 : n1;
}

template <typename WT, int NB>
cudaError_t decode_launch_nb(const DecodeParams &p, int grid, size_t smem, cudaStream_t stream, bool cooperative) {
    void *fn = p.tp > 1 ? reinterpret_cast<void *>(decode_kernel<WT, NB, true>)
                        : reinterpret_cast<void *>(decode_kernel<WT, NB, false>);
    void *args[] = {const_cast<DecodeParams *>(&p)};
    if (cooperative) return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, stream);
    return cudaLaunchKernel(fn, dim3(grid), dim3(kThreads), args, smem, stream);
}

}  // namespace mg

// Explicit instantiation of the host helpers (and so of the kernels) for one row count.
#define MG_DECODE_INSTANTIATE_WT(WT, NB)                                                                       \
    namespace mg {                                                                                             \
    template size_t decode_static_smem_nb<WT, NB>();                                                           \
    template cudaError_t decode_prepare_nb<WT, NB>(size_t);                                                    \
    template int decode_occupancy_nb<WT, NB>(size_t);                                                          \
    template cudaError_t decode_launch_nb<WT, NB>(const DecodeParams &, int, size_t, cudaStream_t, bool);      \
    }
#define MG_DECODE_INSTANTIATE(NB)             \
    MG_DECODE_INSTANTIATE_WT(float, NB)       \
    MG_DECODE_INSTANTIATE_WT(__nv_bfloat16, NB)

// decode.cu -- persistent sm_100a decode kernel for the Gemma 3 forward step.
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
//    of the consumers and across phase boundaries.
//  * Warps 0-7 consume: each phase waits on a gpu-scope counter for its input
//    activations, builds the normalised input vector in shared memory (RMSNorm
//    with (1 + w), residual adds), then multiplies it by the staged tiles with
//    128-bit shared loads and warp-shuffle reductions.
//  * Fusions: input/pre-ff/post-attn/post-ff/final norms and residual adds in
//    the next phase's prologue; QK-norm, RoPE and the K/V write in the attention
//    prologue; GeGLU in the gate/up epilogue; a per-CTA top-k of the lm_head
//    rows in its epilogue; the draw in the last phase.
//  * Attention is split-KV with online softmax; the last CTA to finish a
//    (row, kv head) combines the chunks.
//  * All waits are bounded (common.cuh); on timeout the kernel fast-forwards.
#include "common.cuh"
#include "decode.cuh"
#include "select.cuh"

namespace mg {

// ---------------------------------------------------------------- sync layout
__device__ __forceinline__ uint32_t *ctr_phase(const DecodeParams &p, int ph) { return p.sync + ph; }
__device__ __forceinline__ uint32_t *ctr_att_done(const DecodeParams &p, int l) { return p.sync + p.n_phases + l; }
__device__ __forceinline__ uint32_t *ctr_att_cnt(const DecodeParams &p, int b, int kvh) {
    return p.sync + p.n_phases + p.L + b * p.Hkv + kvh;
}
__device__ __forceinline__ uint32_t *ctr_exit(const DecodeParams &p) {
    return p.sync + p.n_phases + p.L + kMaxRows * p.Hkv;
}

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

template <typename WT>
struct GemvGeom {
    const WT *w1;
    const WT *w2;  // up_proj rows for the gate/up phase, else null
    int64_t row0;
    int nrows, Kp, kc, nseg, rps, ngroups;
};

template <typename WT>
__device__ __forceinline__ void gemv_geom(const DecodeParams &p, int kind, int layer, int ph, GemvGeom<WT> &g) {
    const LayerPtrs &lp = p.layers[layer];
    int N;
    g.w2 = nullptr;
    switch (kind) {
        case PH_QKV:
            N = p.qkv_rows;
            g.Kp = p.Hp;
            g.w1 = static_cast<const WT *>(lp.qkv);
            break;
        case PH_O:
            N = p.H;
            g.Kp = p.Ap;
            g.w1 = static_cast<const WT *>(lp.o);
            break;
        case PH_GU:
            N = p.I;
            g.Kp = p.Hp;
            g.w1 = static_cast<const WT *>(lp.gate);
            g.w2 = static_cast<const WT *>(lp.up);
            break;
        case PH_D:
            N = p.H;
            g.Kp = p.Ip;
            g.w1 = static_cast<const WT *>(lp.down);
            break;
        default:
            N = (p.lm_mode == kLmLogits) ? p.V : 0;
            g.Kp = p.Hp;
            g.w1 = static_cast<const WT *>(p.lm_head);
            break;
    }
    const int slot = cta_slot(ph);
    const int64_t r0 = static_cast<int64_t>(N) * slot / gridDim.x;
    const int64_t r1 = static_cast<int64_t>(N) * (slot + 1) / gridDim.x;
    g.row0 = r0;
    g.nrows = static_cast<int>(r1 - r0);
    constexpr int rpw = sizeof(WT) == 2 ? 2 : 1;
    g.rps = kConsumerWarps * rpw;
    const int mult = g.w2 ? 2 : 1;
    int kc = (kStageBytes / (g.rps * mult * static_cast<int>(sizeof(WT)))) & ~7;
    if (kc > g.Kp) kc = g.Kp;
    g.kc = kc;
    g.nseg = (g.Kp + kc - 1) / kc;
    g.ngroups = (g.nrows + g.rps - 1) / g.rps;
}

// Attention work split: items are (row, kv head, chunk of att_ch positions).
struct AttRows {
    int lo[kMaxRows], n[kMaxRows], nch[kMaxRows];
    int nitems;
};

__device__ __forceinline__ void att_rows(const DecodeParams &p, int layer, const int *s_pos, AttRows &a) {
    const bool global = p.layers[layer].is_global != 0;
    a.nitems = 0;
    for (int b = 0; b < p.B; ++b) {
        const int pos = s_pos[b];
        int lo = 0;
        if (!global && p.window > 0 && pos - p.window + 1 > 0) lo = pos - p.window + 1;
        a.lo[b] = lo;
        a.n[b] = pos + 1 - lo;
        a.nch[b] = (a.n[b] + p.att_ch - 1) / p.att_ch;
        a.nitems += p.Hkv * a.nch[b];
    }
}

__device__ __forceinline__ void att_item(const DecodeParams &p, const AttRows &a, int item, int &b, int &kvh,
                                         int &c) {
    int base = 0;
    b = 0;
    for (; b < p.B; ++b) {
        const int cnt = p.Hkv * a.nch[b];
        if (item < base + cnt) break;
        base += cnt;
    }
    const int r = item - base;
    kvh = r / a.nch[b];
    c = r - kvh * a.nch[b];
}

// ---------------------------------------------------------------- shared memory
struct Smem {
    uint64_t *full;
    uint64_t *empty;
    unsigned char *ring;
    float *xs;  // activation stage / attention scratch / selection scratch
};

struct SmallSmem {
    int pos[kMaxRows];
    int tok[kMaxRows];
    int active[kMaxRows];
    float red[kConsumerWarps * kMaxRows];
    float stat[kMaxRows];
    uint32_t flag;
    uint32_t pad_;
};

// ---------------------------------------------------------------- consumer helpers
// Block sum over consumer threads of one value per row.
__device__ __forceinline__ void block_sum_rows(float (&v)[kMaxRows], int B, SmallSmem &ss, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    for (int b = 0; b < B; ++b) {
        const float s = warp_sum(v[b]);
        if (lane == 0) ss.red[warp * kMaxRows + b] = s;
    }
    consumer_sync(kConsumerThreads);
    for (int b = 0; b < B; ++b) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) t += ss.red[w * kMaxRows + b];
        v[b] = t;
    }
    consumer_sync(kConsumerThreads);
}

// xs[b][0..H) <- rmsnorm(src[b]) * (1 + w); pads [H, Kp) with zeros.
// src rows are read through L2 (written by other CTAs).
__device__ __forceinline__ void stage_rmsnorm(const float *src, int ld, const float *w, int H, int Kp, int B,
                                              float *xs, SmallSmem &ss, int tid) {
    float sq[kMaxRows];
    for (int b = 0; b < B; ++b) {
        float s = 0.f;
        for (int i = tid; i < H; i += kConsumerThreads) {
            const float v = __ldcg(src + static_cast<int64_t>(b) * ld + i);
            xs[b * Kp + i] = v;
            s += v * v;
        }
        sq[b] = s;
    }
    block_sum_rows(sq, B, ss, tid);
    for (int b = 0; b < B; ++b) {
        const float inv = 1.0f / sqrtf(sq[b] / static_cast<float>(H) + 1e-6f);
        for (int i = tid; i < Kp; i += kConsumerThreads)
            xs[b * Kp + i] = i < H ? xs[b * Kp + i] * inv * (1.0f + w[i]) : 0.0f;
    }
    consumer_sync(kConsumerThreads);
}

// x = base + rmsnorm(add) * (1 + w_add), written to xs (unnormalised) and,
// when out != null, to out[b] (the residual stream); then xs <- rmsnorm(x)*(1+w_next).
__device__ __forceinline__ void stage_residual_norm(const float *base, const float *add, const float *w_add,
                                                    const float *w_next, float *out, int H, int Kp, int B,
                                                    float *xs, SmallSmem &ss, int tid) {
    float sq[kMaxRows];
    for (int b = 0; b < B; ++b) {
        float s = 0.f;
        for (int i = tid; i < H; i += kConsumerThreads) {
            const float v = __ldcg(add + static_cast<int64_t>(b) * H + i);
            xs[b * Kp + i] = v;
            s += v * v;
        }
        sq[b] = s;
    }
    block_sum_rows(sq, B, ss, tid);
    float sq2[kMaxRows];
    for (int b = 0; b < B; ++b) {
        const float inv = 1.0f / sqrtf(sq[b] / static_cast<float>(H) + 1e-6f);
        float s = 0.f;
        for (int i = tid; i < H; i += kConsumerThreads) {
            const float x = __ldcg(base + static_cast<int64_t>(b) * H + i) + xs[b * Kp + i] * inv * (1.0f + w_add[i]);
            xs[b * Kp + i] = x;
            if (out) out[static_cast<int64_t>(b) * H + i] = x;
            s += x * x;
        }
        sq2[b] = s;
    }
    block_sum_rows(sq2, B, ss, tid);
    for (int b = 0; b < B; ++b) {
        const float inv = 1.0f / sqrtf(sq2[b] / static_cast<float>(H) + 1e-6f);
        for (int i = tid; i < Kp; i += kConsumerThreads)
            xs[b * Kp + i] = i < H ? xs[b * Kp + i] * inv * (1.0f + w_next[i]) : 0.0f;
    }
    consumer_sync(kConsumerThreads);
}

// Announce this CTA's part of a phase (release at gpu scope).
__device__ __forceinline__ void cta_signal(uint32_t *ctr, int tid) {
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
        __threadfence();
        red_release_add_u32(ctr, 1u);
    }
}

// Wait for a counter; uniform result across consumer threads.
__device__ __forceinline__ bool cta_wait(const uint32_t *ctr, uint32_t target, uint32_t *err, uint32_t site,
                                         SmallSmem &ss, int tid) {
    if (tid == 0) ss.flag = wait_counter_geq(ctr, target, err, site) ? 1u : 0u;
    consumer_sync(kConsumerThreads);
    const bool ok = ss.flag != 0u;
    consumer_sync(kConsumerThreads);
    return ok;
}

// ---------------------------------------------------------------- GEMV consumer
// Multiplies the staged tiles of one phase by xs and hands each finished row's
// per-batch-row dot products to epi(row, b, dot) (dot2 = up row for gate/up).
template <typename WT, class Epi>
__device__ __forceinline__ void gemv_consume(const GemvGeom<WT> &g, int B, const float *xs, const Smem &sm, int S,
                                             uint32_t &tile, uint32_t *err, bool &ok, int tid, Epi epi) {
    constexpr int rpw = sizeof(WT) == 2 ? 2 : 1;
    const int lane = tid & 31, warp = tid >> 5;
    const bool pair = g.w2 != nullptr;
    for (int grp = 0; grp < g.ngroups; ++grp) {
        const int nr = min(g.rps, g.nrows - grp * g.rps);
        float acc[rpw][kMaxRows], acc2[rpw][kMaxRows];
#pragma unroll
        for (int k = 0; k < rpw; ++k)
#pragma unroll
            for (int b = 0; b < kMaxRows; ++b) acc[k][b] = acc2[k][b] = 0.f;
        for (int s = 0; s < g.nseg; ++s, ++tile) {
            const int st = static_cast<int>(tile % S);
            const uint32_t par = (tile / S) & 1u;
            if (ok) ok = mbar_wait(&sm.full[st], par, err, kErrTimeoutFull | 1u);
            const int c0 = s * g.kc;
            const int sw = min(g.kc, g.Kp - c0);
            const WT *stage = reinterpret_cast<const WT *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
            if (ok) {
#pragma unroll
                for (int k = 0; k < rpw; ++k) {
                    const int j = warp * rpw + k;
                    if (j < nr) {
                        const WT *wr = stage + static_cast<size_t>(j) * g.kc;
                        const WT *ur = stage + static_cast<size_t>(g.rps + j) * g.kc;
                        for (int c = lane * 4; c < sw; c += 128) {
                            const float4 w4 = lds_w4(wr + c);
                            float4 u4 = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (pair) u4 = lds_w4(ur + c);
#pragma unroll
                            for (int b = 0; b < kMaxRows; ++b) {
                                if (b < B) {
                                    const float4 x4 = *reinterpret_cast<const float4 *>(xs + b * g.Kp + c0 + c);
                                    acc[k][b] += w4.x * x4.x + w4.y * x4.y + w4.z * x4.z + w4.w * x4.w;
                                    if (pair) acc2[k][b] += u4.x * x4.x + u4.y * x4.y + u4.z * x4.z + u4.w * x4.w;
                                }
                            }
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
            for (int b = 0; b < kMaxRows; ++b) {
                if (b < B) {
                    const float d = warp_sum(acc[k][b]);
                    const float d2 = pair ? warp_sum(acc2[k][b]) : 0.f;
                    if (lane == 0 && j < nr && ok) epi(g.row0 + grp * g.rps + j, b, d, d2);
                }
            }
        }
    }
}

// ---------------------------------------------------------------- the kernel
template <typename WT>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ SmallSmem ss;
    Smem sm;
    {
        uintptr_t base = reinterpret_cast<uintptr_t>(smem_raw);
        base = (base + 127) & ~static_cast<uintptr_t>(127);
        sm.ring = reinterpret_cast<unsigned char *>(base);
        sm.xs = reinterpret_cast<float *>(sm.ring + static_cast<size_t>(p.S) * kStageBytes);
        sm.full = reinterpret_cast<uint64_t *>(sm.xs + p.xs_floats);
        sm.empty = sm.full + p.S;
    }
    const int tid = threadIdx.x;
    const int G = gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < p.S; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
        }
        fence_barrier_init();
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
        if (tok < 0 || tok >= p.V) {
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
    __syncthreads();

    const int warp = tid >> 5;
    if (warp == kConsumerWarps) {
        // ============================ producer ============================
        if ((tid & 31) == 0) {
            const uint64_t pol_w = policy_evict_first();
            uint32_t tile = 0, issued = 0;
            bool ok = true;
            for (int ph = p.ph_begin; ph < p.ph_end; ++ph) {
                int kind, layer;
                phase_of(ph, p.L, kind, layer);
                if (kind == PH_ATT) {
                    AttRows a;
                    att_rows(p, layer, ss.pos, a);
                    const int slot = cta_slot(ph);
                    for (int item = slot; item < a.nitems; item += G) {
                        int b, kvh, c;
                        att_item(p, a, item, b, kvh, c);
                        const int t_begin = a.lo[b] + c * p.att_ch;
                        const int t_end = min(t_begin + p.att_ch, ss.pos[b] + 1);
                        const size_t kvbase = static_cast<size_t>(layer) * p.kv_layer_stride +
                                              static_cast<size_t>(b) * p.kv_row_stride +
                                              static_cast<size_t>(kvh) * p.kv_head_stride;
                        for (int ts = t_begin; ts < t_end; ts += kAttTile, ++tile) {
                            const int st = static_cast<int>(tile % p.S);
                            if (tile >= static_cast<uint32_t>(p.S) && ok)
                                ok = mbar_wait(&sm.empty[st], ((tile / p.S) - 1) & 1u, p.err, kErrTimeoutEmpty | 2u);
                            const int te = min(ts + kAttTile, t_end);
                            const int ncached = max(0, min(te, ss.pos[b]) - ts);
                            const uint32_t bytes = static_cast<uint32_t>(ncached * p.hdp * 4);
                            if (!ok) continue;
                            issued = tile + 1;
                            mbar_arrive_expect_tx(&sm.full[st], 2u * bytes);
                            if (bytes) {
                                unsigned char *dst = sm.ring + static_cast<size_t>(st) * kStageBytes;
                                const size_t off = kvbase + static_cast<size_t>(ts) * p.hdp;
                                bulk_g2s(dst, p.kc + off, bytes, &sm.full[st], pol_w);
                                bulk_g2s(dst + static_cast<size_t>(kAttTile) * p.hdp * 4, p.vc + off, bytes,
                                         &sm.full[st], pol_w);
                            }
                        }
                    }
                } else if (kind != PH_SAMPLE) {
                    GemvGeom<WT> g;
                    gemv_geom<WT>(p, kind, layer, ph, g);
                    const size_t esz = sizeof(WT);
                    for (int grp = 0; grp < g.ngroups; ++grp) {
                        const int nr = min(g.rps, g.nrows - grp * g.rps);
                        const int64_t rbase = g.row0 + static_cast<int64_t>(grp) * g.rps;
                        for (int s = 0; s < g.nseg; ++s, ++tile) {
                            const int st = static_cast<int>(tile % p.S);
                            if (tile >= static_cast<uint32_t>(p.S) && ok)
                                ok = mbar_wait(&sm.empty[st], ((tile / p.S) - 1) & 1u, p.err, kErrTimeoutEmpty | 1u);
                            if (!ok) continue;
                            const int c0 = s * g.kc;
                            const int sw = min(g.kc, g.Kp - c0);
                            const int mult = g.w2 ? 2 : 1;
                            const uint32_t bytes = static_cast<uint32_t>(nr * sw * esz * mult);
                            issued = tile + 1;
                            mbar_arrive_expect_tx(&sm.full[st], bytes);
                            unsigned char *dst = sm.ring + static_cast<size_t>(st) * kStageBytes;
                            if (g.nseg == 1) {
                                const uint32_t blk = static_cast<uint32_t>(nr * g.Kp * esz);
                                bulk_g2s(dst, g.w1 + rbase * g.Kp, blk, &sm.full[st], pol_w);
                                if (g.w2)
                                    bulk_g2s(dst + static_cast<size_t>(g.rps) * g.kc * esz, g.w2 + rbase * g.Kp, blk,
                                             &sm.full[st], pol_w);
                            } else {
                                for (int j = 0; j < nr; ++j) {
                                    bulk_g2s(dst + static_cast<size_t>(j) * g.kc * esz, g.w1 + (rbase + j) * g.Kp + c0,
                                             static_cast<uint32_t>(sw * esz), &sm.full[st], pol_w);
                                    if (g.w2)
                                        bulk_g2s(dst + static_cast<size_t>(g.rps + j) * g.kc * esz,
                                                 g.w2 + (rbase + j) * g.Kp + c0, static_cast<uint32_t>(sw * esz),
                                                 &sm.full[st], pol_w);
                                }
                            }
                        }
                    }
                }
            }
            // Drain: copies still in flight must land before the CTA exits.
            const uint32_t first = issued > static_cast<uint32_t>(p.S) ? issued - p.S : 0u;
            for (uint32_t t = first; t < issued; ++t) {
                if (!mbar_wait_drain(&sm.full[t % p.S], (t / p.S) & 1u)) set_error(p.err, kErrTimeoutDrain);
            }
        }
    } else {
        // ============================ consumers ============================
        bool ok = ld_relaxed_u32(p.err) == 0u;
        uint32_t tile = 0;
        const int lane = tid & 31;
        const int B = p.B;
        for (int ph = p.ph_begin; ph < p.ph_end; ++ph) {
            int kind, layer;
            phase_of(ph, p.L, kind, layer);
            const LayerPtrs &lp = p.layers[layer];
            if (kind == PH_QKV) {
                if (layer > 0 && ph - 1 >= p.ph_begin)
                    ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                GemvGeom<WT> g;
                gemv_geom<WT>(p, kind, layer, ph, g);
                float *out_h = (blockIdx.x == 0) ? p.h : nullptr;
                if (layer == 0) {
                    // embedding row * sqrt(H) (model.mojo:62-68, layers.mojo:247-251)
                    const float scale = sqrtf(static_cast<float>(p.H));
                    const WT *E = static_cast<const WT *>(p.embed);
                    for (int b = 0; b < B; ++b)
                        for (int i = tid; i < p.H; i += kConsumerThreads) {
                            const float x = ld_w(E + static_cast<int64_t>(ss.tok[b]) * p.embed_ld + i) * scale;
                            sm.xs[b * g.Kp + i] = x;
                            if (out_h) out_h[static_cast<int64_t>(b) * p.H + i] = x;
                        }
                    consumer_sync(kConsumerThreads);
                    // in-place norm of xs
                    float sq[kMaxRows];
                    for (int b = 0; b < B; ++b) {
                        float s = 0.f;
                        for (int i = tid; i < p.H; i += kConsumerThreads) {
                            const float v = sm.xs[b * g.Kp + i];
                            s += v * v;
                        }
                        sq[b] = s;
                    }
                    block_sum_rows(sq, B, ss, tid);
                    for (int b = 0; b < B; ++b) {
                        const float inv = 1.0f / sqrtf(sq[b] / static_cast<float>(p.H) + 1e-6f);
                        for (int i = tid; i < g.Kp; i += kConsumerThreads)
                            sm.xs[b * g.Kp + i] = i < p.H ? sm.xs[b * g.Kp + i] * inv * (1.0f + lp.in_ln[i]) : 0.f;
                    }
                    consumer_sync(kConsumerThreads);
                } else {
                    const LayerPtrs &prev = p.layers[layer - 1];
                    stage_residual_norm(p.r, p.mlp_raw, prev.post_ff_ln, lp.in_ln, out_h, p.H, g.Kp, B, sm.xs, ss,
                                        tid);
                }
                float *qkv = p.qkv;
                const int ld = p.qkv_rows;
                gemv_consume<WT>(g, B, sm.xs, sm, p.S, tile, p.err, ok, tid,
                                 [&](int64_t row, int b, float d, float) { qkv[static_cast<int64_t>(b) * ld + row] = d; });
                cta_signal(ctr_phase(p, ph), tid);
            } else if (kind == PH_ATT) {
                if (ph - 1 >= p.ph_begin) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                AttRows a;
                att_rows(p, layer, ss.pos, a);
                const int Gq = p.Hq / p.Hkv;
                const int hd = p.hd;
                const int half = hd / 2;
                // attention scratch in xs: q [Gq][hd], knew [hd], vnew [hd], sc [Gq][kAttTile], m/l/alpha [Gq]
                float *q_s = sm.xs;
                float *k_s = q_s + Gq * hd;
                float *v_s = k_s + hd;
                float *sc = v_s + hd;
                float *m_s = sc + Gq * kAttTile;
                float *l_s = m_s + kMaxQPerKv;
                float *al_s = l_s + kMaxQPerKv;
                int *flag_s = reinterpret_cast<int *>(al_s + kMaxQPerKv);
                const float scale = 1.0f / sqrtf(static_cast<float>(hd));
                const int slot = cta_slot(ph);
                for (int item = slot; item < a.nitems; item += G) {
                    int b, kvh, c;
                    att_item(p, a, item, b, kvh, c);
                    const int pos = ss.pos[b];
                    const int t_begin = a.lo[b] + c * p.att_ch;
                    const int t_end = min(t_begin + p.att_ch, pos + 1);
                    const float *cosr = (lp.is_global ? p.rope_cos_g : p.rope_cos_l) + static_cast<int64_t>(pos) * half;
                    const float *sinr = (lp.is_global ? p.rope_sin_g : p.rope_sin_l) + static_cast<int64_t>(pos) * half;
                    // ---- prologue: QK-norm + RoPE of this group's q heads and the new k; new v.
                    const float *qkv_b = p.qkv + static_cast<int64_t>(b) * p.qkv_rows;
                    for (int vec = warp; vec < Gq + 2; vec += kConsumerWarps) {
                        const float *src;
                        float *dst;
                        const float *nw;
                        bool rope = true;
                        if (vec < Gq) {
                            src = qkv_b + static_cast<int64_t>(kvh * Gq + vec) * hd;
                            dst = q_s + vec * hd;
                            nw = lp.q_norm;
                        } else if (vec == Gq) {
                            src = qkv_b + p.A + static_cast<int64_t>(kvh) * hd;
                            dst = k_s;
                            nw = lp.k_norm;
                        } else {
                            src = qkv_b + p.A + static_cast<int64_t>(p.Hkv + kvh) * hd;
                            dst = v_s;
                            nw = nullptr;
                            rope = false;
                        }
                        float s = 0.f;
                        for (int d = lane; d < hd; d += 32) {
                            const float v = __ldcg(src + d);
                            dst[d] = v;
                            s += v * v;
                        }
                        s = warp_sum(s);
                        if (nw) {
                            const float inv = 1.0f / sqrtf(s / static_cast<float>(hd) + 1e-6f);
                            for (int d = lane; d < hd; d += 32) dst[d] = dst[d] * inv * (1.0f + nw[d]);
                        }
                        __syncwarp();
                        if (rope) {
                            for (int i = lane; i < half; i += 32) {
                                const float x1 = dst[i], x2 = dst[i + half];
                                const float cs = cosr[i], sn = sinr[i];
                                dst[i] = x1 * cs - x2 * sn;
                                dst[i + half] = x2 * cs + x1 * sn;
                            }
                        }
                        __syncwarp();
                    }
                    if (tid < Gq) {
                        m_s[tid] = -INFINITY;
                        l_s[tid] = 0.f;
                    }
                    consumer_sync(kConsumerThreads);
                    // K/V write at pos by the chunk that ends there (layers.mojo:57-61).
                    if (t_end == pos + 1 && ss.active[b] && ok) {
                        const size_t off = static_cast<size_t>(layer) * p.kv_layer_stride +
                                           static_cast<size_t>(b) * p.kv_row_stride +
                                           static_cast<size_t>(kvh) * p.kv_head_stride + static_cast<size_t>(pos) * p.hdp;
                        for (int d = tid; d < hd; d += kConsumerThreads) {
                            p.kc[off + d] = k_s[d];
                            p.vc[off + d] = v_s[d];
                        }
                    }
                    float acc[kMaxQPerKv * kMaxHeadDim / kConsumerThreads];
#pragma unroll
                    for (int j = 0; j < kMaxQPerKv * kMaxHeadDim / kConsumerThreads; ++j) acc[j] = 0.f;
                    const int nout = Gq * hd;
                    for (int ts = t_begin; ts < t_end; ts += kAttTile, ++tile) {
                        const int st = static_cast<int>(tile % p.S);
                        if (ok) ok = mbar_wait(&sm.full[st], (tile / p.S) & 1u, p.err, kErrTimeoutFull | 2u);
                        const int nt = min(kAttTile, t_end - ts);
                        const float *kt = reinterpret_cast<const float *>(sm.ring + static_cast<size_t>(st) * kStageBytes);
                        const float *vt = kt + kAttTile * p.hdp;
                        // scores
                        for (int pr = warp; pr < Gq * nt; pr += kConsumerWarps) {
                            const int h = pr / nt, t = pr - h * nt;
                            const float *kr = (ts + t == pos) ? k_s : kt + t * p.hdp;
                            const float *qr = q_s + h * hd;
                            float s = 0.f;
                            for (int d = lane; d < hd; d += 32) s += qr[d] * kr[d];
                            s = warp_sum(s);
                            if (lane == 0) sc[h * kAttTile + t] = s * scale;
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
                        // P @ V
#pragma unroll
                        for (int j = 0; j < kMaxQPerKv * kMaxHeadDim / kConsumerThreads; ++j) {
                            const int o = tid + j * kConsumerThreads;
                            if (o < nout) {
                                const int h = o / hd, d = o - h * hd;
                                float a2 = acc[j] * al_s[h];
                                for (int t = 0; t < nt; ++t) {
                                    const float vv = (ts + t == pos) ? v_s[d] : vt[t * p.hdp + d];
                                    a2 += sc[h * kAttTile + t] * vv;
                                }
                                acc[j] = a2;
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sm.empty[st]);
                        consumer_sync(kConsumerThreads);
                    }
                    // ---- partial (m, l, acc) for this chunk
                    const int part_ld = hd + 2;
                    float *part = p.attn_part +
                                  ((static_cast<int64_t>(b) * p.Hkv + kvh) * p.max_ch + c) * Gq * part_ld;
#pragma unroll
                    for (int j = 0; j < kMaxQPerKv * kMaxHeadDim / kConsumerThreads; ++j) {
                        const int o = tid + j * kConsumerThreads;
                        if (o < nout) {
                            const int h = o / hd, d = o - h * hd;
                            part[h * part_ld + 2 + d] = acc[j];
                        }
                    }
                    if (tid < Gq) {
                        part[tid * part_ld + 0] = m_s[tid];
                        part[tid * part_ld + 1] = l_s[tid];
                    }
                    consumer_sync(kConsumerThreads);
                    if (tid == 0) {
                        __threadfence();
                        const uint32_t old = atomicAdd(ctr_att_cnt(p, b, kvh), 1u);
                        flag_s[0] = (old + 1u == static_cast<uint32_t>(a.nch[b])) ? 1 : 0;
                    }
                    consumer_sync(kConsumerThreads);
                    if (flag_s[0]) {
                        // last chunk to finish: combine all chunks of (b, kvh)
                        __threadfence();
                        const int nch = a.nch[b];
                        const float *pb = p.attn_part + (static_cast<int64_t>(b) * p.Hkv + kvh) * p.max_ch * Gq * part_ld;
                        // per head: M and 1/L into m_s / l_s
                        for (int h = warp; h < Gq; h += kConsumerWarps) {
                            float mx = -INFINITY;
                            for (int cc = lane; cc < nch; cc += 32) mx = fmaxf(mx, __ldcg(pb + (cc * Gq + h) * part_ld));
                            mx = warp_max(mx);
                            float lsum = 0.f;
                            for (int cc = lane; cc < nch; cc += 32) {
                                const float mc = __ldcg(pb + (cc * Gq + h) * part_ld);
                                lsum += __ldcg(pb + (cc * Gq + h) * part_ld + 1) * expf(mc - mx);
                            }
                            lsum = warp_sum(lsum);
                            if (lane == 0) {
                                m_s[h] = mx;
                                l_s[h] = 1.0f / lsum;
                            }
                        }
                        consumer_sync(kConsumerThreads);
                        float *ao = p.attn_out + static_cast<int64_t>(b) * p.Ap + static_cast<int64_t>(kvh) * Gq * hd;
                        for (int o = tid; o < nout; o += kConsumerThreads) {
                            const int h = o / hd, d = o - h * hd;
                            float sacc = 0.f;
                            for (int cc = 0; cc < nch; ++cc) {
                                const float *pc = pb + (cc * Gq + h) * part_ld;
                                sacc += __ldcg(pc + 2 + d) * expf(__ldcg(pc) - m_s[h]);
                            }
                            ao[o] = sacc * l_s[h];
                        }
                        consumer_sync(kConsumerThreads);
                        if (tid == 0) {
                            *ctr_att_cnt(p, b, kvh) = 0u;
                            __threadfence();
                            red_release_add_u32(ctr_att_done(p, layer), 1u);
                        }
                    }
                    consumer_sync(kConsumerThreads);
                }
            } else if (kind == PH_O) {
                if (ph - 1 >= p.ph_begin)
                    ok = cta_wait(ctr_att_done(p, layer), static_cast<uint32_t>(B * p.Hkv), p.err, 100 + ph, ss, tid) &&
                         ok;
                GemvGeom<WT> g;
                gemv_geom<WT>(p, kind, layer, ph, g);
                for (int b = 0; b < B; ++b)
                    for (int i = tid; i < g.Kp; i += kConsumerThreads)
                        sm.xs[b * g.Kp + i] = __ldcg(p.attn_out + static_cast<int64_t>(b) * p.Ap + i);
                consumer_sync(kConsumerThreads);
                float *o_raw = p.o_raw;
                const int H = p.H;
                gemv_consume<WT>(g, B, sm.xs, sm, p.S, tile, p.err, ok, tid,
                                 [&](int64_t row, int b, float d, float) { o_raw[static_cast<int64_t>(b) * H + row] = d; });
                cta_signal(ctr_phase(p, ph), tid);
            } else if (kind == PH_GU) {
                if (ph - 1 >= p.ph_begin) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                GemvGeom<WT> g;
                gemv_geom<WT>(p, kind, layer, ph, g);
                // r = h + norm(o_raw, post_attn) (layers.mojo:202-207); xs = norm(r, pre_ff) (209-210)
                stage_residual_norm(p.h, p.o_raw, lp.post_attn_ln, lp.pre_ff_ln, blockIdx.x == 0 ? p.r : nullptr,
                                    p.H, g.Kp, B, sm.xs, ss, tid);
                float *act = p.act;
                const int Ip = p.Ip;
                const float sqrt_2 = 1.4142135623730951f;
                gemv_consume<WT>(g, B, sm.xs, sm, p.S, tile, p.err, ok, tid, [&](int64_t row, int b, float gd, float ud) {
                    const float gelu = 0.5f * gd * (1.0f + erff(gd / sqrt_2));  // ops.mojo:19-22
                    act[static_cast<int64_t>(b) * Ip + row] = gelu * ud;
                });
                cta_signal(ctr_phase(p, ph), tid);
            } else if (kind == PH_D) {
                if (ph - 1 >= p.ph_begin) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                GemvGeom<WT> g;
                gemv_geom<WT>(p, kind, layer, ph, g);
                for (int b = 0; b < B; ++b)
                    for (int i = tid; i < g.Kp; i += kConsumerThreads)
                        sm.xs[b * g.Kp + i] = __ldcg(p.act + static_cast<int64_t>(b) * p.Ip + i);
                consumer_sync(kConsumerThreads);
                float *mlp = p.mlp_raw;
                const int H = p.H;
                gemv_consume<WT>(g, B, sm.xs, sm, p.S, tile, p.err, ok, tid,
                                 [&](int64_t row, int b, float d, float) { mlp[static_cast<int64_t>(b) * H + row] = d; });
                cta_signal(ctr_phase(p, ph), tid);
            } else if (kind == PH_LMH) {
                if (ph - 1 >= p.ph_begin) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                GemvGeom<WT> g;
                gemv_geom<WT>(p, kind, layer, ph, g);
                if (p.lm_mode != kLmNone) {
                    // x = r + norm(mlp_raw, post_ff); xs = norm(x, final norm) (layers.mojo:283-285)
                    stage_residual_norm(p.r, p.mlp_raw, lp.post_ff_ln, p.final_norm, nullptr, p.H, g.Kp, B, sm.xs, ss,
                                        tid);
                }
                if (p.lm_mode == kLmEmbed) {
                    if (blockIdx.x == 0 && ok)
                        for (int b = 0; b < B; ++b)
                            if (ss.active[b])
                                for (int i = tid; i < p.H; i += kConsumerThreads)
                                    p.emb_acc[static_cast<int64_t>(b) * p.H + i] += sm.xs[b * g.Kp + i];
                } else if (p.lm_mode == kLmLogits) {
                    float *logits = p.logits;
                    const int V = p.V;
                    gemv_consume<WT>(g, B, sm.xs, sm, p.S, tile, p.err, ok, tid, [&](int64_t row, int b, float d, float) {
                        logits[static_cast<int64_t>(b) * V + row] = d;
                    });
                    if (p.topk > 0) {
                        consumer_sync(kConsumerThreads);
                        SelectSmem &sel = *reinterpret_cast<SelectSmem *>(sm.xs);
                        uint64_t *outk = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(sm.xs) +
                                                                      sizeof(SelectSmem));
                        for (int b = 0; b < B; ++b) {
                            const float *lr = logits + static_cast<int64_t>(b) * V + g.row0;
                            const uint32_t r0 = static_cast<uint32_t>(g.row0);
                            block_select_topk(
                                g.nrows, p.topk, [&](int i) { return topk_key(lr[i], r0 + static_cast<uint32_t>(i)); },
                                outk, sel, tid, kConsumerThreads, [] { consumer_sync(kConsumerThreads); });
                            uint64_t *dst = p.cand_key + (static_cast<int64_t>(b) * G + blockIdx.x) * kMaxTopK;
                            for (int j = tid; j < p.topk; j += kConsumerThreads) dst[j] = outk[j];
                            consumer_sync(kConsumerThreads);
                        }
                    }
                }
                cta_signal(ctr_phase(p, ph), tid);
            } else {  // PH_SAMPLE
                const int b = blockIdx.x;
                if (b < B) {
                    int32_t token = -1;
                    if (p.sample && p.lm_mode == kLmLogits && p.topk > 0) {
                        if (ph - 1 >= p.ph_begin) ok = cta_wait(ctr_phase(p, ph - 1), G, p.err, 100 + ph, ss, tid) && ok;
                        SelectSmem &sel = *reinterpret_cast<SelectSmem *>(sm.xs);
                        unsigned char *after = reinterpret_cast<unsigned char *>(sm.xs) + sizeof(SelectSmem);
                        uint64_t *outk = reinterpret_cast<uint64_t *>(after);
                        double *fscr = reinterpret_cast<double *>(after + kMaxTopK * sizeof(uint64_t));
                        int *oscr = reinterpret_cast<int *>(fscr + kMaxTopK);
                        const uint64_t *ck = p.cand_key + static_cast<int64_t>(b) * G * kMaxTopK;
                        const int K = p.topk;
                        block_select_topk(
                            G * K, K, [&](int i) { return __ldcg(ck + (i / K) * kMaxTopK + (i % K)); }, outk, sel, tid,
                            kConsumerThreads, [] { consumer_sync(kConsumerThreads); });
                        if (tid == 0 && ok) {
                            const double u = p.uniforms ? p.uniforms[b] : philox_uniform(p.seed, p.rng_offset, b);
                            token = draw_from_sorted(outk, K, p.temperature, p.top_p, u, fscr, oscr);
                        }
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

    // ---- exit: the last CTA out resets the counters used by this launch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(ctr_exit(p), 1u);
        if (old == static_cast<uint32_t>(G - 1)) {
            __threadfence();
            for (int ph = p.ph_begin; ph < p.ph_end; ++ph) *ctr_phase(p, ph) = 0u;
            for (int l = 0; l < p.L; ++l) *ctr_att_done(p, l) = 0u;
            *ctr_exit(p) = 0u;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------- host launch
size_t decode_smem_bytes(int S, int xs_floats) {
    return 128 + static_cast<size_t>(S) * kStageBytes + static_cast<size_t>(xs_floats) * 4 + 2 * S * 8;
}

// Static shared memory of the kernel (SmallSmem) in bytes.
template <typename WT>
size_t decode_static_smem() {
    cudaFuncAttributes a;
    if (cudaFuncGetAttributes(&a, decode_kernel<WT>) != cudaSuccess) return 1024;
    return a.sharedSizeBytes;
}

template <typename WT>
cudaError_t decode_prepare(size_t dynamic_smem) {
    return cudaFuncSetAttribute(decode_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(dynamic_smem));
}

template <typename WT>
int decode_occupancy(size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<WT>, kThreads, smem) != cudaSuccess) return 0;
    return n;
}

template <typename WT>
cudaError_t decode_launch(const DecodeParams &p, int grid, size_t smem, cudaStream_t stream, bool cooperative) {
    if (cooperative) {
        void *args[] = {const_cast<DecodeParams *>(&p)};
        return cudaLaunchCooperativeKernel(reinterpret_cast<void *>(decode_kernel<WT>), dim3(grid), dim3(kThreads),
                                           args, smem, stream);
    }
    decode_kernel<WT><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template size_t decode_static_smem<float>();
template size_t decode_static_smem<__nv_bfloat16>();
template cudaError_t decode_prepare<float>(size_t);
template cudaError_t decode_prepare<__nv_bfloat16>(size_t);
template int decode_occupancy<float>(size_t);
template int decode_occupancy<__nv_bfloat16>(size_t);
template cudaError_t decode_launch<float>(const DecodeParams &, int, size_t, cudaStream_t, bool);
template cudaError_t decode_launch<__nv_bfloat16>(const DecodeParams &, int, size_t, cudaStream_t, bool);

}  // namespace mg

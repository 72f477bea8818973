// prefill.cu -- the batched prefill path: every prompt token of every row in
// one pass per layer, with the projections as tcgen05 GEMMs (gemm_tc.cu) and
// these kernels around them.  Same arithmetic as the decode kernel apart from
// the projections, whose inputs are rounded to bf16 for the tensor cores.
//
// Per layer, for the N packed tokens (row b(n), position pos(n)):
//   xn  = bf16(rmsnorm(x) (1 + in_ln))                      pf_resnorm
//   qkv = xn . Wqkv^T                                       GEMM
//   QK-norm + RoPE of q and k, k and v into the KV cache    pf_qk_rope_kv
//   a   = bf16(causal softmax(q k^T / sqrt(hd)) v)          pf_attention
//   o   = a . Wo^T                                          GEMM
//   r   = x + rmsnorm(o) (1 + post_attn); xn = bf16(rmsnorm(r) (1 + pre_ff))   pf_resnorm
//   gu  = xn . [Wgate; Wup]^T                               GEMM
//   act = bf16(gelu_erf(g) u)                               pf_geglu
//   m   = act . Wdown^T                                     GEMM
//   x   = r + rmsnorm(m) (1 + post_ff)  (and the next layer's xn)             pf_resnorm
// (layers.mojo:174-220 for the layer, 16-97 attention, 101-118 MLP.)
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "decode.cuh"

namespace mg {

constexpr int kPfThreads = 256;

__device__ __forceinline__ float block_sum_pf(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kPfThreads / 32; ++w) t += red[w];
    return t;
}

// x = E[tok] * sqrt(H) (model.mojo:62-68, layers.mojo:247-251)
template <typename ET>
__global__ void __launch_bounds__(kPfThreads) pf_embed_kernel(const ET *E, int64_t ld, const int32_t *tok, int H,
                                                              float scale, float *x) {
    const int n = blockIdx.x;
    const ET *e = E + static_cast<int64_t>(tok[n]) * ld;
    for (int i = threadIdx.x; i < H; i += kPfThreads) x[static_cast<int64_t>(n) * H + i] = ld_w(e + i) * scale;
}

// res = base + (add ? rmsnorm(add) (1 + w_add) : 0);  xn = bf16(rmsnorm(res) (1 + w_next)), zero padded to Kp.
// res may alias base.  One CTA per token.
__global__ void __launch_bounds__(kPfThreads) pf_resnorm_kernel(const float *base, const float *add,
                                                                const float *w_add, const float *w_next, float *res,
                                                                __nv_bfloat16 *xn, int H, int Kp, float inv_h) {
    __shared__ float red[kPfThreads / 32];
    const int64_t n = blockIdx.x;
    const float *b = base + n * H;
    float inv_a = 0.f;
    if (add) {
        float s = 0.f;
        for (int i = threadIdx.x; i < H; i += kPfThreads) {
            const float v = add[n * H + i];
            s += v * v;
        }
        inv_a = rms_inv(block_sum_pf(s, red), inv_h);
    }
    float s2 = 0.f;
    for (int i = threadIdx.x; i < H; i += kPfThreads) {
        float x = b[i];
        if (add) x += add[n * H + i] * inv_a * (1.0f + w_add[i]);
        res[n * H + i] = x;
        s2 += x * x;
    }
    const float inv = rms_inv(block_sum_pf(s2, red), inv_h);
    for (int i = threadIdx.x; i < Kp; i += kPfThreads)
        xn[n * Kp + i] = __float2bfloat16_rn(i < H ? res[n * H + i] * inv * (1.0f + w_next[i]) : 0.f);
}

// The same, one warp per token (8 tokens per CTA), float4 loads; H and Kp multiples of 4.
__global__ void __launch_bounds__(kPfThreads) pf_resnorm_warp_kernel(const float *base, const float *add,
                                                                     const float *w_add, const float *w_next,
                                                                     float *res, __nv_bfloat16 *xn, int H, int Kp,
                                                                     float inv_h, int N) {
    const int lane = threadIdx.x & 31;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * (kPfThreads / 32) + (threadIdx.x >> 5);
    if (n >= N) return;
    const int H4 = H / 4;
    const float4 *b4 = reinterpret_cast<const float4 *>(base + n * H);
    const float4 *a4 = add ? reinterpret_cast<const float4 *>(add + n * H) : nullptr;
    float4 *r4 = reinterpret_cast<float4 *>(res + n * H);
    float inv_a = 0.f;
    if (add) {
        float s = 0.f;
        for (int i = lane; i < H4; i += 32) {
            const float4 v = a4[i];
            s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        inv_a = rms_inv(warp_sum(s), inv_h);
    }
    float s2 = 0.f;
    for (int i = lane; i < H4; i += 32) {
        float4 x = b4[i];
        if (add) {
            const float4 a = a4[i], w = reinterpret_cast<const float4 *>(w_add)[i];
            x.x += a.x * inv_a * (1.0f + w.x);
            x.y += a.y * inv_a * (1.0f + w.y);
            x.z += a.z * inv_a * (1.0f + w.z);
            x.w += a.w * inv_a * (1.0f + w.w);
        }
        r4[i] = x;
        s2 += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    const float inv = rms_inv(warp_sum(s2), inv_h);
    for (int i = lane; i < Kp / 4; i += 32) {
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < H4) {
            const float4 x = r4[i], w = reinterpret_cast<const float4 *>(w_next)[i];
            y = make_float4(x.x * inv * (1.0f + w.x), x.y * inv * (1.0f + w.y), x.z * inv * (1.0f + w.z),
                            x.w * inv * (1.0f + w.w));
        }
        const __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&lo);
        pk.y = *reinterpret_cast<const uint32_t *>(&hi);
        reinterpret_cast<uint2 *>(xn + n * Kp)[i] = pk;
    }
}

// The same for a few tokens (a batched decode step): one CTA per token, every
// load of the row issued before the first reduction (H <= 4 kPfThreads float4s).
__global__ void __launch_bounds__(kPfThreads) pf_resnorm_row_kernel(const float *base, const float *add,
                                                                    const float *w_add, const float *w_next,
                                                                    float *res, __nv_bfloat16 *xn, int H, int Kp,
                                                                    float inv_h) {
    constexpr int kJ = 4;
    __shared__ float red[kPfThreads / 32];
    const int64_t n = blockIdx.x;
    const int H4 = H / 4;
    const float4 *b4 = reinterpret_cast<const float4 *>(base + n * H);
    const float4 *a4 = add ? reinterpret_cast<const float4 *>(add + n * H) : nullptr;
    float4 x[kJ], a[kJ], wa[kJ], wn[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
        const int i = threadIdx.x + j * kPfThreads;
        const bool on = i < H4;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        x[j] = on ? b4[i] : z;
        a[j] = (on && add) ? a4[i] : z;
        wa[j] = (on && add) ? reinterpret_cast<const float4 *>(w_add)[i] : z;
        wn[j] = on ? reinterpret_cast<const float4 *>(w_next)[i] : z;
    }
    if (add) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kJ; ++j) s += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
        const float inv_a = rms_inv(block_sum_pf(s, red), inv_h);
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            x[j].x += a[j].x * inv_a * (1.0f + wa[j].x);
            x[j].y += a[j].y * inv_a * (1.0f + wa[j].y);
            x[j].z += a[j].z * inv_a * (1.0f + wa[j].z);
            x[j].w += a[j].w * inv_a * (1.0f + wa[j].w);
        }
    }
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
        const int i = threadIdx.x + j * kPfThreads;
        if (i < H4) reinterpret_cast<float4 *>(res + n * H)[i] = x[j];
        s2 += x[j].x * x[j].x + x[j].y * x[j].y + x[j].z * x[j].z + x[j].w * x[j].w;
    }
    const float inv = rms_inv(block_sum_pf(s2, red), inv_h);
    for (int i = threadIdx.x; i < Kp / 4; i += kPfThreads) {
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            if (i == static_cast<int>(threadIdx.x) + j * kPfThreads && i < H4)
                y = make_float4(x[j].x * inv * (1.0f + wn[j].x), x[j].y * inv * (1.0f + wn[j].y),
                                x[j].z * inv * (1.0f + wn[j].z), x[j].w * inv * (1.0f + wn[j].w));
        }
        const __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&lo);
        pk.y = *reinterpret_cast<const uint32_t *>(&hi);
        reinterpret_cast<uint2 *>(xn + n * Kp)[i] = pk;
    }
}

// QK-norm (layers.mojo:43-49) and RoPE (52-55) of each token's q heads (in
// place) and k head(s); k and v into the KV cache at (row, pos) (57-61).
// One warp per (token, head vector), 8 per CTA.
__global__ void __launch_bounds__(kPfThreads) pf_qk_rope_kv_kernel(
    float *qkv, int qkv_ld, int Hq, int Hkv, int hd, int hdp, const float *q_norm, const float *k_norm,
    const float *cos_t, const float *sin_t, const int32_t *row, const int32_t *pos, float *kc, float *vc,
    int64_t kv_row_stride, int64_t kv_head_stride, float inv_hd, __nv_bfloat16 *qb, __nv_bfloat16 *kb,
    __nv_bfloat16 *vt, int64_t vt_ld, int N) {
    const int lane = threadIdx.x & 31;
    const int nv = Hq + Hkv;
    const int64_t item = static_cast<int64_t>(blockIdx.x) * (kPfThreads / 32) + (threadIdx.x >> 5);
    if (item >= static_cast<int64_t>(N) * nv) return;
    const int64_t n = item / nv;
    const int half = hd / 2;
    const int p = pos[n];
    float *x0 = qkv + n * qkv_ld;
    {
        const int vec = static_cast<int>(item - n * nv);
        float *x = x0 + static_cast<int64_t>(vec) * hd;  // q heads then k heads (layout of the qkv rows)
        const float *nw = vec < Hq ? q_norm : k_norm;
        if (nw) {
            float s = 0.f;
            for (int d = lane; d < hd; d += 32) s += x[d] * x[d];
            const float inv = rms_inv(warp_sum(s), inv_hd);
            for (int d = lane; d < hd; d += 32) x[d] = x[d] * inv * (1.0f + nw[d]);
            __syncwarp();
        }
        const float *c = cos_t + static_cast<int64_t>(p) * half;
        const float *sn = sin_t + static_cast<int64_t>(p) * half;
        for (int i = lane; i < half; i += 32) {
            const float x1 = x[i], x2 = x[i + half];
            x[i] = x1 * c[i] - x2 * sn[i];
            x[i + half] = x2 * c[i] + x1 * sn[i];
        }
        __syncwarp();
        if (vec >= Hq) {
            const int kvh = vec - Hq;
            const int64_t off = row[n] * kv_row_stride + kvh * kv_head_stride + static_cast<int64_t>(p) * hdp;
            const float *v = x0 + static_cast<int64_t>(Hq + Hkv + kvh) * hd;
            for (int d = lane; d < hd; d += 32) {
                kc[off + d] = x[d];
                vc[off + d] = v[d];
            }
            if (kb) {  // bf16 operands of the tensor-core attention: K by token, V transposed
                for (int d = lane; d < hd; d += 32) {
                    kb[(n * Hkv + kvh) * hd + d] = __float2bfloat16_rn(x[d]);
                    vt[(static_cast<int64_t>(kvh) * hd + d) * vt_ld + n] = __float2bfloat16_rn(v[d]);
                }
            }
        } else if (qb) {
            for (int d = lane; d < hd; d += 32) qb[(n * Hq + vec) * hd + d] = __float2bfloat16_rn(x[d]);
        }
    }
}

// The same for head dims 64 / 128 / 256 with each head vector in registers
// (lane holds dims lane + 32 i; the RoPE partner d + hd/2 is in the same lane).
// Writes only what the attention that follows reads: q / k back into qkv and
// K / V into the cache (kc non-null) for the CUDA-core attention or a later
// decode step, bf16 Q and K (qb, kb non-null) for the tensor-core attention.
template <int HD>
__global__ void __launch_bounds__(kPfThreads) pf_qk_rope_reg_kernel(
    float *qkv, int qkv_ld, int Hq, int Hkv, int hdp, const float *q_norm, const float *k_norm, const float *cos_t,
    const float *sin_t, const int32_t *row, const int32_t *pos, float *kc, float *vc, int64_t kv_row_stride,
    int64_t kv_head_stride, float inv_hd, int write_back, __nv_bfloat16 *qb, __nv_bfloat16 *kb, int N) {
    constexpr int kR = HD / 32, kHalf = HD / 2, kP = kR / 2;
    const int lane = threadIdx.x & 31;
    const int nv = Hq + Hkv;
    const int64_t item = static_cast<int64_t>(blockIdx.x) * (kPfThreads / 32) + (threadIdx.x >> 5);
    if (item >= static_cast<int64_t>(N) * nv) return;
    const int64_t n = item / nv;
    const int vec = static_cast<int>(item - n * nv);
    const int p = pos[n];
    float *x0 = qkv + n * qkv_ld;
    float *xg = x0 + static_cast<int64_t>(vec) * HD;  // q heads then k heads (layout of the qkv rows)
    float x[kR];
#pragma unroll
    for (int i = 0; i < kR; ++i) x[i] = xg[lane + 32 * i];
    const float *nw = vec < Hq ? q_norm : k_norm;
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kR; ++i) ss += x[i] * x[i];
        const float inv = rms_inv(warp_sum(ss), inv_hd);
#pragma unroll
        for (int i = 0; i < kR; ++i) x[i] = x[i] * inv * (1.0f + nw[lane + 32 * i]);
    }
    const float *c = cos_t + static_cast<int64_t>(p) * kHalf;
    const float *sn = sin_t + static_cast<int64_t>(p) * kHalf;
#pragma unroll
    for (int i = 0; i < kP; ++i) {
        const float cc = c[lane + 32 * i], ss = sn[lane + 32 * i];
        const float x1 = x[i], x2 = x[i + kP];
        x[i] = x1 * cc - x2 * ss;
        x[i + kP] = x2 * cc + x1 * ss;
    }
    if (write_back) {
#pragma unroll
        for (int i = 0; i < kR; ++i) xg[lane + 32 * i] = x[i];
    }
    if (vec >= Hq) {
        const int kvh = vec - Hq;
        if (kc) {
            const int64_t off = row[n] * kv_row_stride + kvh * kv_head_stride + static_cast<int64_t>(p) * hdp;
            const float *v = x0 + static_cast<int64_t>(Hq + Hkv + kvh) * HD;
#pragma unroll
            for (int i = 0; i < kR; ++i) {
                kc[off + lane + 32 * i] = x[i];
                vc[off + lane + 32 * i] = v[lane + 32 * i];
            }
        }
        if (kb) {
#pragma unroll
            for (int i = 0; i < kR; ++i) kb[(n * Hkv + kvh) * HD + lane + 32 * i] = __float2bfloat16_rn(x[i]);
        }
    } else if (qb) {
#pragma unroll
        for (int i = 0; i < kR; ++i) qb[(n * Hq + vec) * HD + lane + 32 * i] = __float2bfloat16_rn(x[i]);
    }
}

// vt[c][n] = bf16(V[n][c]) for the packed tokens (V = the v part of the qkv
// rows, c over Hkv * hd): 32 x 32 tiles through shared memory, so both the
// reads (along c) and the writes (along n) are coalesced.
__global__ void __launch_bounds__(kPfThreads) pf_v_transpose_kernel(const float *qkv, int qkv_ld, int v_off, int C,
                                                                    __nv_bfloat16 *vt, int64_t vt_ld, int N) {
    __shared__ float tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    const int n0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
#pragma unroll
    for (int r = ty; r < 32; r += kPfThreads / 32) {
        const int n = n0 + r, c = c0 + tx;
        tile[r][tx] = (n < N && c < C) ? qkv[static_cast<int64_t>(n) * qkv_ld + v_off + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int r = ty; r < 32; r += kPfThreads / 32) {
        const int c = c0 + r, n = n0 + tx;
        if (c < C && n < N) vt[static_cast<int64_t>(c) * vt_ld + n] = __float2bfloat16_rn(tile[tx][r]);
    }
}

// Causal attention over the cached positions lo..pos (layers.mojo:63-94).  One
// CTA per (token, kv head) for its GQ q heads (each K/V row read once for the
// group); its 8 warps take interleaved blocks of 32 keys, one key per lane:
// a lane forms its key's GQ scores over the whole head (q in shared memory,
// read as a broadcast), a warp-wide max/sum per head updates that warp's
// online softmax, and P.V runs with lanes over head dims.  The warps' partial
// (m, l, acc) are combined in shared memory.
// Split-KV (kchunk > 0, few tokens such as a batched decode step): blockIdx.y
// takes keys [lo + y kchunk, lo + (y + 1) kchunk) and the CTA writes its
// (m, l, unnormalised acc) per q head to part; pf_attn_combine_kernel merges.
template <int GQ>
__global__ void __launch_bounds__(kPfThreads) pf_attention_kernel(
    const float *qkv, int qkv_ld, int Hq, int Hkv, int hd, int hdp, const float *kc, const float *vc,
    const int32_t *row, const int32_t *pos, const int32_t *last, int64_t kv_row_stride, int64_t kv_head_stride,
    int window, int is_global, float scale, __nv_bfloat16 *out, int out_ld, int N, int kchunk, float *part) {
    constexpr int kQ = GQ > 0 ? GQ : kMaxQPerKv;
    constexpr int kDL = kMaxHeadDim / 32;
    constexpr int kW = kPfThreads / 32;
    extern __shared__ __align__(16) float sm_dyn[];  // q [gq][hd] | acc [kW][gq][hd] | m, l [kW][gq]
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int gq = GQ > 0 ? GQ : Hq / Hkv;
    const int64_t n = blockIdx.x / Hkv;
    const int kvh = static_cast<int>(blockIdx.x - n * Hkv);
    float *qs = sm_dyn;
    float *pacc = qs + gq * hd;
    float *pm = pacc + kW * gq * hd;
    float *pl = pm + kW * gq;
    const int p = pos[n];
    const int lo = (!is_global && window > 0 && p - window + 1 > 0) ? p - window + 1 : 0;
    // causal: keys up to the token itself; with `last` (an encoder): up to the
    // sequence's last token, within the symmetric window on local layers
    int hi = p;
    if (last) {
        hi = last[n];
        if (!is_global && window > 0) hi = min(hi, p + window - 1);
    }
    const float *q = qkv + n * qkv_ld + static_cast<int64_t>(kvh) * gq * hd;
    for (int i = threadIdx.x; i < gq * hd; i += kPfThreads) qs[i] = q[i];
    __syncthreads();
    const float *kb = kc + row[n] * kv_row_stride + kvh * kv_head_stride;
    const float *vb = vc + row[n] * kv_row_stride + kvh * kv_head_stride;
    float m[kQ], l[kQ], acc[kQ][kDL];
#pragma unroll
    for (int h = 0; h < kQ; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < kDL; ++i) acc[h][i] = 0.f;
    }
    int klo = lo, khi = hi;
    if (kchunk > 0) {
        klo = lo + static_cast<int>(blockIdx.y) * kchunk;
        khi = min(hi, klo + kchunk - 1);
    }
    for (int t0 = klo + 32 * w; t0 <= khi; t0 += 32 * kW) {
        const int t = t0 + lane;
        const bool valid = t <= hi;
        float s[kQ];
#pragma unroll
        for (int h = 0; h < kQ; ++h) s[h] = 0.f;
        if (valid) {
            const float4 *k4 = reinterpret_cast<const float4 *>(kb + static_cast<int64_t>(t) * hdp);
            for (int d4 = 0; d4 < hd / 4; ++d4) {
                const float4 kv = k4[d4];
#pragma unroll
                for (int h = 0; h < kQ; ++h) {
                    if (h < gq) {
                        const float4 qv = *reinterpret_cast<const float4 *>(qs + h * hd + 4 * d4);
                        s[h] += qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
                    }
                }
            }
        }
        float pr[kQ];
#pragma unroll
        for (int h = 0; h < kQ; ++h) {
            if (h < gq) {
                const float sh = valid ? s[h] * scale : -INFINITY;
                const float m_new = fmaxf(m[h], warp_max(sh));
                const float alpha = (m[h] == -INFINITY) ? 0.f : expf(m[h] - m_new);
                pr[h] = valid ? expf(sh - m_new) : 0.f;
                l[h] = l[h] * alpha + warp_sum(pr[h]);
#pragma unroll
                for (int i = 0; i < kDL; ++i) acc[h][i] *= alpha;
                m[h] = m_new;
            }
        }
        const int nb = min(32, hi - t0 + 1);
        for (int j = 0; j < nb; ++j) {
            const float *v = vb + static_cast<int64_t>(t0 + j) * hdp;
            float vv[kDL];
#pragma unroll
            for (int i = 0; i < kDL; ++i) {
                const int d = lane + 32 * i;
                vv[i] = d < hd ? v[d] : 0.f;
            }
#pragma unroll
            for (int h = 0; h < kQ; ++h) {
                if (h < gq) {
                    const float pj = __shfl_sync(0xffffffffu, pr[h], j);
#pragma unroll
                    for (int i = 0; i < kDL; ++i) acc[h][i] += pj * vv[i];
                }
            }
        }
    }
    // combine the warps' partials
#pragma unroll
    for (int h = 0; h < kQ; ++h) {
        if (h < gq) {
            if (lane == 0) {
                pm[w * gq + h] = m[h];
                pl[w * gq + h] = l[h];
            }
#pragma unroll
            for (int i = 0; i < kDL; ++i) {
                const int d = lane + 32 * i;
                if (d < hd) pacc[(w * gq + h) * hd + d] = acc[h][i];
            }
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < gq * hd; e += kPfThreads) {
        const int h = e / hd, d = e - h * hd;
        float M = -INFINITY;
#pragma unroll
        for (int u = 0; u < kW; ++u) M = fmaxf(M, pm[u * gq + h]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int u = 0; u < kW; ++u) {
            const float mu = pm[u * gq + h];
            if (mu == -INFINITY) continue;  // a warp that saw no key
            const float f = expf(mu - M);
            L += pl[u * gq + h] * f;
            o += pacc[(u * gq + h) * hd + d] * f;
        }
        if (part) {  // [N * Hkv][splits][gq][2 + hd]: m, l, acc
            float *pp = part + ((static_cast<int64_t>(blockIdx.x) * gridDim.y + blockIdx.y) * gq + h) * (hd + 2);
            if (d == 0) {
                pp[0] = M;
                pp[1] = L;
            }
            pp[2 + d] = M == -INFINITY ? 0.f : o;
        } else {
            out[n * out_ld + static_cast<int64_t>(kvh * gq + h) * hd + d] = __float2bfloat16_rn(o / L);
        }
    }
}

// Decode-shaped split of the attention (one query per (token, kv head), a key
// range per blockIdx.y, as pf_attention_kernel with kchunk > 0): lanes run over
// head dims, so every key row is one coalesced warp load; each warp takes keys
// four at a time (interleaved with the other warps) and keeps its own online
// softmax per q head; the 8 warps merge in shared memory and the CTA writes
// its split's (m, l, unnormalised acc) to part for pf_attn_combine_kernel.
template <int GQ, int HD>
__global__ void __launch_bounds__(kPfThreads) pf_attn_decode_kernel(
    const float *qkv, int qkv_ld, int Hkv, int hdp, const float *kc, const float *vc, const int32_t *row,
    const int32_t *pos, int64_t kv_row_stride, int64_t kv_head_stride, int window, int is_global, float scale,
    int kchunk, float *part) {
    constexpr int kW = kPfThreads / 32;
    constexpr int kJ = (HD + 127) / 128;  // float4 of a head row per lane
    constexpr int kB = 4;                 // keys per warp step
    __shared__ float sm_m[kW][GQ], sm_l[kW][GQ];
    __shared__ __align__(16) float sm_acc[kW][GQ][HD];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t n = blockIdx.x / Hkv;
    const int kvh = static_cast<int>(blockIdx.x - n * Hkv);
    const int p = pos[n];
    const int lo = (!is_global && window > 0 && p - window + 1 > 0) ? p - window + 1 : 0;
    const int klo = lo + static_cast<int>(blockIdx.y) * kchunk;
    const int khi = min(p, klo + kchunk - 1);
    const float *qb = qkv + n * qkv_ld + static_cast<int64_t>(kvh) * GQ * HD;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 q[GQ][kJ];
#pragma unroll
    for (int h = 0; h < GQ; ++h)
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            const int f = lane + 32 * j;
            q[h][j] = 4 * f < HD ? *reinterpret_cast<const float4 *>(qb + h * HD + 4 * f) : z4;
        }
    const int64_t kvoff = row[n] * kv_row_stride + kvh * kv_head_stride;
    const float *kb = kc + kvoff, *vb = vc + kvoff;
    float m[GQ], l[GQ];
    float4 acc[GQ][kJ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int j = 0; j < kJ; ++j) acc[h][j] = z4;
    }
    for (int t0 = klo + w * kB; t0 <= khi; t0 += kW * kB) {
        float4 kr[kB][kJ], vr[kB][kJ];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            const int t = t0 + b;
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int f = lane + 32 * j;
                const bool on = t <= khi && 4 * f < HD;
                kr[b][j] = on ? *reinterpret_cast<const float4 *>(kb + static_cast<int64_t>(t) * hdp + 4 * f) : z4;
                vr[b][j] = on ? *reinterpret_cast<const float4 *>(vb + static_cast<int64_t>(t) * hdp + 4 * f) : z4;
            }
        }
        float sc[kB][GQ];
#pragma unroll
        for (int b = 0; b < kB; ++b)
#pragma unroll
            for (int h = 0; h < GQ; ++h) {
                float a = 0.f;
#pragma unroll
                for (int j = 0; j < kJ; ++j)
                    a += q[h][j].x * kr[b][j].x + q[h][j].y * kr[b][j].y + q[h][j].z * kr[b][j].z +
                         q[h][j].w * kr[b][j].w;
                sc[b][h] = a;
            }
#pragma unroll
        for (int b = 0; b < kB; ++b)
#pragma unroll
            for (int h = 0; h < GQ; ++h) sc[b][h] = t0 + b <= khi ? warp_sum(sc[b][h]) * scale : -INFINITY;
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
            float mx = sc[0][h];
#pragma unroll
            for (int b = 1; b < kB; ++b) mx = fmaxf(mx, sc[b][h]);
            const float m_new = fmaxf(m[h], mx);
            const float alpha = m[h] == -INFINITY ? 0.f : expf(m[h] - m_new);
            float pb[kB], ps = 0.f;
#pragma unroll
            for (int b = 0; b < kB; ++b) {
                pb[b] = sc[b][h] == -INFINITY ? 0.f : expf(sc[b][h] - m_new);
                ps += pb[b];
            }
            l[h] = l[h] * alpha + ps;
            m[h] = m_new;
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                float4 a = acc[h][j];
                a.x *= alpha;
                a.y *= alpha;
                a.z *= alpha;
                a.w *= alpha;
#pragma unroll
                for (int b = 0; b < kB; ++b) {
                    a.x += pb[b] * vr[b][j].x;
                    a.y += pb[b] * vr[b][j].y;
                    a.z += pb[b] * vr[b][j].z;
                    a.w += pb[b] * vr[b][j].w;
                }
                acc[h][j] = a;
            }
        }
    }
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
        if (lane == 0) {
            sm_m[w][h] = m[h];
            sm_l[w][h] = l[h];
        }
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            const int f = lane + 32 * j;
            if (4 * f < HD) *reinterpret_cast<float4 *>(&sm_acc[w][h][4 * f]) = acc[h][j];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < GQ * HD; e += kPfThreads) {
        const int h = e / HD, d = e - h * HD;
        float M = -INFINITY;
#pragma unroll
        for (int u = 0; u < kW; ++u) M = fmaxf(M, sm_m[u][h]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int u = 0; u < kW; ++u) {
            if (sm_m[u][h] == -INFINITY) continue;  // a warp that saw no key
            const float f = expf(sm_m[u][h] - M);
            L += sm_l[u][h] * f;
            o += sm_acc[u][h][d] * f;
        }
        float *pp = part + ((static_cast<int64_t>(blockIdx.x) * gridDim.y + blockIdx.y) * GQ + h) * (HD + 2);
        if (d == 0) {
            pp[0] = M;
            pp[1] = L;
        }
        pp[2 + d] = M == -INFINITY ? 0.f : o;
    }
}

// out[n][(kvh gq + h) hd + d] from the splits' (m, l, acc) of (token n, kv head kvh).
__global__ void __launch_bounds__(kPfThreads) pf_attn_combine_kernel(const float *part, int splits, int gq, int hd,
                                                                     int Hkv, __nv_bfloat16 *out, int out_ld) {
    const int64_t n = blockIdx.x / Hkv;
    const int kvh = static_cast<int>(blockIdx.x - n * Hkv);
    const float *base = part + static_cast<int64_t>(blockIdx.x) * splits * gq * (hd + 2);
    for (int e = threadIdx.x; e < gq * hd; e += kPfThreads) {
        const int h = e / hd, d = e - h * hd;
        float M = -INFINITY;
        for (int y = 0; y < splits; ++y) M = fmaxf(M, base[(y * gq + h) * (hd + 2)]);
        float L = 0.f, o = 0.f;
        for (int y = 0; y < splits; ++y) {
            const float *pp = base + (y * gq + h) * (hd + 2);
            if (pp[0] == -INFINITY) continue;  // a split with no key in range
            const float f = expf(pp[0] - M);
            L += pp[1] * f;
            o += pp[2 + d] * f;
        }
        out[n * out_ld + static_cast<int64_t>(kvh * gq + h) * hd + d] = __float2bfloat16_rn(o / L);
    }
}

// act = bf16(gelu_erf(gate) * up) (ops.mojo:5-30); gu rows hold [gate (I) | up (I)].
// il: gate and up columns in alternating blocks of 128 (feature f at column
// 256 (f / 128) + f % 128, its up value 128 further) instead of [gate | up].
__device__ __forceinline__ int geglu_gate_col(int f, int il) { return il ? ((f & ~127) << 1) + (f & 127) : f; }

__global__ void __launch_bounds__(kPfThreads) pf_geglu_kernel(const float *gu, int I, int gu_ld, __nv_bfloat16 *act,
                                                              int Ip, int il) {
    const int64_t n = blockIdx.x;
    for (int i = blockIdx.y * kPfThreads + threadIdx.x; i < Ip; i += gridDim.y * kPfThreads) {
        float a = 0.f;
        if (i < I) {
            const int gc = geglu_gate_col(i, il), uc = il ? gc + 128 : I + i;
            const float g = gu[n * gu_ld + gc], u = gu[n * gu_ld + uc];
            a = 0.5f * g * (1.0f + erff(g * kInvSqrt2)) * u;
        }
        act[n * Ip + i] = __float2bfloat16_rn(a);
    }
}
// The same, 4 features per thread (I, Ip and gu_ld multiples of 4).
__global__ void __launch_bounds__(kPfThreads) pf_geglu4_kernel(const float *gu, int I, int gu_ld, __nv_bfloat16 *act,
                                                               int Ip, int il) {
    const int64_t n = blockIdx.x;
    const int i = 4 * (blockIdx.y * kPfThreads + threadIdx.x);
    if (i >= Ip) return;
    float r[4] = {0.f, 0.f, 0.f, 0.f};
    if (i < I) {
        const int gc = geglu_gate_col(i, il), uc = il ? gc + 128 : I + i;  // 4 features stay in one block
        const float4 g = *reinterpret_cast<const float4 *>(gu + n * gu_ld + gc);
        const float4 u = *reinterpret_cast<const float4 *>(gu + n * gu_ld + uc);
        r[0] = 0.5f * g.x * (1.0f + erff(g.x * kInvSqrt2)) * u.x;
        r[1] = 0.5f * g.y * (1.0f + erff(g.y * kInvSqrt2)) * u.y;
        r[2] = 0.5f * g.z * (1.0f + erff(g.z * kInvSqrt2)) * u.z;
        r[3] = 0.5f * g.w * (1.0f + erff(g.w * kInvSqrt2)) * u.w;
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(r[0], r[1]), hi = __floats2bfloat162_rn(r[2], r[3]);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t *>(&lo);
    pk.y = *reinterpret_cast<const uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(act + n * Ip + i) = pk;
}

// ---- encoder head: pooling, dense layers, L2 normalisation
// inv[t] = 1 / rms(x_t) over the packed tokens, one warp per token.
__global__ void __launch_bounds__(kPfThreads) pf_rowinv_kernel(const float *x, int H, float inv_h, float *inv,
                                                               int N) {
    const int t = blockIdx.x * (kPfThreads / 32) + (threadIdx.x >> 5);
    if (t >= N) return;
    const float *xt = x + static_cast<int64_t>(t) * H;
    float s = 0.f;
    for (int i = threadIdx.x & 31; i < H; i += 32) s += xt[i] * xt[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) inv[t] = rms_inv(s, inv_h);
}
// pool[b][i] = mean over the sequence's tokens [start[b], start[b] + len[b]) of
// x_t[i] inv[t] (1 + w[i]) -- the final norm (layers.mojo:283-285) then the
// mean, in fp32.  Grid (sequences, column blocks of kPfThreads).
__global__ void __launch_bounds__(kPfThreads) pf_pool_kernel(const float *x, int H, const int32_t *start,
                                                             const int32_t *len, const float *w, const float *inv,
                                                             float *pool) {
    const int b = blockIdx.x;
    const int i = blockIdx.y * kPfThreads + threadIdx.x;
    if (i >= H) return;
    float acc = 0.f;
    for (int t = start[b]; t < start[b] + len[b]; ++t) acc += x[static_cast<int64_t>(t) * H + i] * inv[t];
    pool[static_cast<int64_t>(b) * H + i] = acc * (1.0f + w[i]) / static_cast<float>(len[b]);
}

// out[b][o] = sum_k W[o][k] in[b][k] (fp32), one warp per (b, o).
__global__ void __launch_bounds__(kPfThreads) pf_dense_kernel(const float *in, int K, const float *W, int O,
                                                              float *out, int B) {
    const int lane = threadIdx.x & 31;
    const int64_t task = static_cast<int64_t>(blockIdx.x) * (kPfThreads / 32) + (threadIdx.x >> 5);
    if (task >= static_cast<int64_t>(B) * O) return;
    const int64_t b = task / O, o = task - b * O;
    const float *xi = in + b * K, *wr = W + o * K;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += wr[k] * xi[k];
    s = warp_sum(s);
    if (lane == 0) out[b * O + o] = s;
}

// row b scaled to unit L2 norm.
__global__ void __launch_bounds__(kPfThreads) pf_l2norm_kernel(float *y, int H) {
    __shared__ float red[kPfThreads / 32];
    float *r = y + static_cast<int64_t>(blockIdx.x) * H;
    float s = 0.f;
    for (int i = threadIdx.x; i < H; i += kPfThreads) s += r[i] * r[i];
    const float inv = rsqrtf(fmaxf(block_sum_pf(s, red), 1e-24f));
    for (int i = threadIdx.x; i < H; i += kPfThreads) r[i] *= inv;
}

// ---------------------------------------------------------------- launches
cudaError_t pf_encoder_head(const float *x, int H, int N, const int32_t *start, const int32_t *len,
                            const float *final_norm, float inv_h, float *row_inv, const float *d0, int d0_out,
                            const float *d1, float *pool, float *mid, float *out, int B, cudaStream_t s) {
    constexpr int wpb = kPfThreads / 32;
    pf_rowinv_kernel<<<(N + wpb - 1) / wpb, kPfThreads, 0, s>>>(x, H, inv_h, row_inv, N);
    pf_pool_kernel<<<dim3(B, (H + kPfThreads - 1) / kPfThreads), kPfThreads, 0, s>>>(x, H, start, len, final_norm,
                                                                                       row_inv, d0 ? pool : out);
    if (d0) {
        const int w = kPfThreads / 32;
        pf_dense_kernel<<<static_cast<int>((static_cast<int64_t>(B) * d0_out + w - 1) / w), kPfThreads, 0, s>>>(
            pool, H, d0, d0_out, mid, B);
        pf_dense_kernel<<<static_cast<int>((static_cast<int64_t>(B) * H + w - 1) / w), kPfThreads, 0, s>>>(
            mid, d0_out, d1, H, out, B);
    }
    pf_l2norm_kernel<<<B, kPfThreads, 0, s>>>(out, H);
    return cudaGetLastError();
}
cudaError_t pf_embed(const void *E, int wdtype_bf16, int64_t ld, const int32_t *tok, int N, int H, float scale,
                     float *x, cudaStream_t s) {
    if (wdtype_bf16)
        pf_embed_kernel<__nv_bfloat16><<<N, kPfThreads, 0, s>>>(static_cast<const __nv_bfloat16 *>(E), ld, tok, H,
                                                                  scale, x);
    else
        pf_embed_kernel<float><<<N, kPfThreads, 0, s>>>(static_cast<const float *>(E), ld, tok, H, scale, x);
    return cudaGetLastError();
}
cudaError_t pf_resnorm(const float *base, const float *add, const float *w_add, const float *w_next, float *res,
                       __nv_bfloat16 *xn, int N, int H, int Kp, float inv_h, cudaStream_t s) {
    if (H % 4 == 0 && Kp % 4 == 0 && N < 8 * 148 && H <= 16 * kPfThreads)
        pf_resnorm_row_kernel<<<N, kPfThreads, 0, s>>>(base, add, w_add, w_next, res, xn, H, Kp, inv_h);
    else if (H % 4 == 0 && Kp % 4 == 0)
        pf_resnorm_warp_kernel<<<(N + kPfThreads / 32 - 1) / (kPfThreads / 32), kPfThreads, 0, s>>>(
            base, add, w_add, w_next, res, xn, H, Kp, inv_h, N);
    else
        pf_resnorm_kernel<<<N, kPfThreads, 0, s>>>(base, add, w_add, w_next, res, xn, H, Kp, inv_h);
    return cudaGetLastError();
}
// q/k norm + RoPE, the cache write (kc null: skipped; only for the
// tensor-core attention of an encoder pass) and the bf16 operands of the
// tensor-core attention (qb null: none, and q / k go back into qkv for the
// CUDA-core attention).
cudaError_t pf_qk_rope_kv(float *qkv, int qkv_ld, int N, int Hq, int Hkv, int hd, int hdp, const float *q_norm,
                          const float *k_norm, const float *cos_t, const float *sin_t, const int32_t *row,
                          const int32_t *pos, float *kc, float *vc, int64_t kv_row_stride, int64_t kv_head_stride,
                          float inv_hd, __nv_bfloat16 *qb, __nv_bfloat16 *kb, __nv_bfloat16 *vt, int64_t vt_ld,
                          cudaStream_t s) {
    const int64_t items = static_cast<int64_t>(N) * (Hq + Hkv);
    const unsigned blocks = static_cast<unsigned>((items + kPfThreads / 32 - 1) / (kPfThreads / 32));
    if (hd == 64 || hd == 128 || hd == 256) {
        const int write_back = qb ? 0 : 1;
#define MG_PF_ROPE(HD)                                                                                            \
    pf_qk_rope_reg_kernel<HD><<<blocks, kPfThreads, 0, s>>>(qkv, qkv_ld, Hq, Hkv, hdp, q_norm, k_norm, cos_t,     \
                                                            sin_t, row, pos, kc, vc, kv_row_stride,             \
                                                            kv_head_stride, inv_hd, write_back, qb, kb, N)
        if (hd == 64) MG_PF_ROPE(64);
        else if (hd == 128) MG_PF_ROPE(128);
        else MG_PF_ROPE(256);
#undef MG_PF_ROPE
        if (vt) {
            const dim3 g((N + 31) / 32, (Hkv * hd + 31) / 32);
            pf_v_transpose_kernel<<<g, kPfThreads, 0, s>>>(qkv, qkv_ld, (Hq + Hkv) * hd, Hkv * hd, vt, vt_ld, N);
        }
        return cudaGetLastError();
    }
    if (!kc) return cudaErrorInvalidValue;  // the generic kernel always fills the cache
    pf_qk_rope_kv_kernel<<<static_cast<unsigned>((items + kPfThreads / 32 - 1) / (kPfThreads / 32)), kPfThreads, 0,
                           s>>>(qkv, qkv_ld, Hq, Hkv, hd, hdp, q_norm, k_norm, cos_t, sin_t, row,
                                                    pos, kc, vc, kv_row_stride, kv_head_stride, inv_hd, qb, kb, vt,
                                                    vt_ld, N);
    return cudaGetLastError();
}
cudaError_t pf_attention(const float *qkv, int qkv_ld, int N, int Hq, int Hkv, int hd, int hdp, const float *kc,
                         const float *vc, const int32_t *row, const int32_t *pos, const int32_t *last,
                         int64_t kv_row_stride, int64_t kv_head_stride, int window, int is_global, float scale,
                         __nv_bfloat16 *out, int out_ld, int max_ctx, float *ws, size_t ws_floats, cudaStream_t s) {
    const int blocks = N * Hkv;
    // few (token, kv head) pairs and long contexts: split the keys so the grid
    // covers about two waves of SMs (blocks of 64+ keys), then merge
    int splits = 1, kchunk = 0;
    if (ws && blocks < 148 && max_ctx > 128) {
        splits = std::min((max_ctx + 63) / 64, std::max(1, 2 * 148 / blocks));
        kchunk = (max_ctx + splits - 1) / splits;
        kchunk = (kchunk + 31) / 32 * 32;
        splits = (max_ctx + kchunk - 1) / kchunk;
        if (static_cast<size_t>(blocks) * splits * (Hq / Hkv) * (hd + 2) > ws_floats) splits = 1, kchunk = 0;
    }
    float *part = splits > 1 ? ws : nullptr;
    if (splits == 1) kchunk = 0;
    const int gq = Hq / Hkv;
    const size_t smem = sizeof(float) * (static_cast<size_t>(gq) * hd * (1 + kPfThreads / 32) + 2 * (kPfThreads / 32) * gq);
#define MG_PF_ATT(G)                                                                                                \
    do {                                                                                                            \
        if (smem > 48 * 1024) {                                                                                     \
            const cudaError_t e = cudaFuncSetAttribute(pf_attention_kernel<G>,                                      \
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                                                       static_cast<int>(smem));                                     \
            if (e != cudaSuccess) return e;                                                                         \
        }                                                                                                           \
        pf_attention_kernel<G><<<dim3(blocks, splits), kPfThreads, smem, s>>>(                                      \
            qkv, qkv_ld, Hq, Hkv, hd, hdp, kc, vc, row, pos, last, kv_row_stride, kv_head_stride, window, is_global,  \
            scale, out, out_ld, N, kchunk, part);                                                                   \
    } while (0)
    bool done = false;
    if (part) {  // decode-shaped split: coalesced key rows
#define MG_PF_DEC(G, HD_)                                                                                           \
    if (gq == G && hd == HD_) {                                                                                     \
        pf_attn_decode_kernel<G, HD_><<<dim3(blocks, splits), kPfThreads, 0, s>>>(                                  \
            qkv, qkv_ld, Hkv, hdp, kc, vc, row, pos, kv_row_stride, kv_head_stride, window, is_global, scale, kchunk, \
            part);                                                                                                  \
        done = true;                                                                                                \
    }
        MG_PF_DEC(1, 256) MG_PF_DEC(2, 256) MG_PF_DEC(3, 256) MG_PF_DEC(4, 256)
        MG_PF_DEC(1, 128) MG_PF_DEC(2, 128) MG_PF_DEC(4, 128)
        MG_PF_DEC(1, 64) MG_PF_DEC(2, 64) MG_PF_DEC(4, 64)
#undef MG_PF_DEC
    }
    if (!done) {
        switch (Hq / Hkv) {
            case 1: MG_PF_ATT(1); break;
            case 2: MG_PF_ATT(2); break;
            case 4: MG_PF_ATT(4); break;
            default: MG_PF_ATT(0); break;
        }
    }
#undef MG_PF_ATT
    if (part)
        pf_attn_combine_kernel<<<blocks, kPfThreads, 0, s>>>(part, splits, Hq / Hkv, hd, Hkv, out, out_ld);
    return cudaGetLastError();
}
// pos[b] += 1 for rows [0, n): the positions after a batched decode step.
__global__ void pf_advance_kernel(int32_t *pos, int n) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n) pos[b] += 1;
}
cudaError_t pf_advance(int32_t *pos, int n, cudaStream_t s) {
    pf_advance_kernel<<<(n + 127) / 128, 128, 0, s>>>(pos, n);
    return cudaGetLastError();
}
cudaError_t pf_geglu(const float *gu, int I, int gu_ld, __nv_bfloat16 *act, int Ip, int N, int il, cudaStream_t s) {
    if (I % 4 == 0 && Ip % 4 == 0 && gu_ld % 4 == 0)
        pf_geglu4_kernel<<<dim3(N, (Ip / 4 + kPfThreads - 1) / kPfThreads), kPfThreads, 0, s>>>(gu, I, gu_ld, act, Ip,
                                                                                               il);
    else
        pf_geglu_kernel<<<dim3(N, (Ip + kPfThreads - 1) / kPfThreads), kPfThreads, 0, s>>>(gu, I, gu_ld, act, Ip, il);
    return cudaGetLastError();
}

}  // namespace mg

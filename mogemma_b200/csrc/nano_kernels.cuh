// nano_kernels.cuh -- kernels of the Gemma 3n ("nano") decode step.
//
// Restates, on the device, forward_nano_step (src/mo/mogemma/layers.mojo:
// 959-1004) and what it calls (373-956, 121-171).  The step is a fixed chain of
// small kernels -- GEMVs with one warp per output row, single-CTA norms and
// AltUp mixing, one CTA per head for attention -- captured once into a CUDA
// graph and replayed per token: the position and the token are read from
// device memory, so the same graph serves every step.  No kernel waits on
// another CTA, so nothing can hang.  fp32 throughout, as the reference.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace mg {
namespace nano {

constexpr int kBlock = 256;          // threads of the single-CTA kernels
constexpr int kWarpsPerGemv = 8;     // output rows per GEMV block
constexpr int kMaxModalities = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Sum over a block of kBlock threads (red: kBlock / 32 floats of shared memory).
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kBlock / 32; ++w) t += red[w];
    return t;
}
__device__ __forceinline__ float block_max(float v, float *red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = -INFINITY;
#pragma unroll
    for (int w = 0; w < kBlock / 32; ++w) t = fmaxf(t, red[w]);
    return t;
}

// out[o] = scale * sum_i W[o][i] x[i]  (vec_mat_mul, ops.mojo:69-95; W row-major [out][in]).
// One warp per row; float4 loads when the row length is a multiple of 4.
__global__ void __launch_bounds__(kWarpsPerGemv * 32) k_gemv(float *__restrict__ out, const float *__restrict__ x,
                                                             const float *__restrict__ W, int in, int out_dim,
                                                             float scale) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarpsPerGemv + (threadIdx.x >> 5);
    if (row >= out_dim) return;
    const float *wr = W + static_cast<int64_t>(row) * in;
    float acc = 0.f;
    if ((in & 3) == 0) {
        const float4 *w4 = reinterpret_cast<const float4 *>(wr);
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (int i = lane; i < in / 4; i += 32) {
            const float4 a = __ldg(w4 + i), b = x4[i];
            acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
        }
    } else {
        for (int i = lane; i < in; i += 32) acc += __ldg(wr + i) * x[i];
    }
    acc = warp_sum(acc);
    if (lane == 0) out[row] = acc * scale;
}

// out = x / sqrt(mean(x^2) + eps) * w (or unit weights when w is null), optionally plus base
// (_rms_norm_nano_weighted / _unit, layers.mojo:373-401).  One CTA; out may alias x.
__global__ void __launch_bounds__(kBlock) k_rms(float *out, const float *x, const float *w, const float *base, int n) {
    __shared__ float red[kBlock / 32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += kBlock) s += x[i] * x[i];
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(s / static_cast<float>(n) + 1e-6f);
    for (int i = threadIdx.x; i < n; i += kBlock) {
        float v = x[i] * inv;
        if (w) v *= w[i];
        if (base) v = base[i] + v;
        out[i] = v;
    }
}

// Token embedding * sqrt(H) into stream 0 (layers.mojo:877-881).
__global__ void k_embed(float *stream0, const float *E, const int32_t *tok, int H, float scale) {
    const int64_t t = *tok;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        stream0[i] = E[t * H + i] * scale;
}

// Streams 1.. scaled to the base stream's magnitude (_prepare_altup_streams, layers.mojo:633-657):
// stream[k] = proj[k - 1] * mag(base) / max(mag(proj[k - 1]), 1e-6), one CTA per projected stream.
__global__ void __launch_bounds__(kBlock) k_match_magnitude(float *streams, const float *proj, int H) {
    __shared__ float red[kBlock / 32];
    const int k = blockIdx.x + 1;
    const float *p = proj + static_cast<int64_t>(blockIdx.x) * H;
    float sb = 0.f, sp = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlock) {
        sb += streams[i] * streams[i];
        sp += p[i] * p[i];
    }
    sb = block_sum(sb, red);
    sp = block_sum(sp, red);
    const float target = sqrtf(sb / static_cast<float>(H) + 1e-6f);
    const float pm = fmaxf(sqrtf(sp / static_cast<float>(H) + 1e-6f), 1e-6f);
    const float scale = target / pm;
    for (int i = threadIdx.x; i < H; i += kBlock) streams[static_cast<int64_t>(k) * H + i] = p[i] * scale;
}

// Per-layer input projection (layers.mojo:674-681): proj[l][p] = sum_d base[d] W[d][l][p] / sqrt(H),
// W [H][T][P]; one thread per (l, p), consecutive threads on consecutive p (coalesced).
__global__ void k_ple_project(float *proj, const float *base, const float *W, int H, int T, int P, int L, float scale) {
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= L * P) return;
    const int l = o / P, p = o - l * P;
    const float *wc = W + static_cast<int64_t>(l) * P + p;
    const int64_t stride = static_cast<int64_t>(T) * P;
    float acc = 0.f;
    for (int d = 0; d < H; ++d) acc += base[d] * __ldg(wc + d * stride);
    proj[o] = acc * scale;
}

// Per layer l (one CTA each): pli[l] = (norm_w(proj[l]) + table[tok][l] * sqrt(P)) / sqrt(2)
// (layers.mojo:683-693).
__global__ void __launch_bounds__(kBlock) k_ple_finish(float *pli, const float *proj, const float *norm_w,
                                                       const float *table, const int32_t *tok, int T, int P) {
    __shared__ float red[kBlock / 32];
    const int l = blockIdx.x;
    const float *pr = proj + static_cast<int64_t>(l) * P;
    float s = 0.f;
    for (int i = threadIdx.x; i < P; i += kBlock) s += pr[i] * pr[i];
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(s / static_cast<float>(P) + 1e-6f);
    const float es = sqrtf(static_cast<float>(P));
    const float *tb = table + (static_cast<int64_t>(*tok) * T + l) * P;
    for (int i = threadIdx.x; i < P; i += kBlock)
        pli[static_cast<int64_t>(l) * P + i] = (pr[i] * inv * norm_w[i] + tb[i] * es) * 0.7071067811865475f;
}

// tanh(router . (norm_w(x) / H)) (_compute_router_modalities, layers.mojo:525-542), into mod[nm].
__device__ void router_modalities(float *mod, const float *x, const float *router, const float *router_norm, int H,
                                  int nm, float *red) {
    float s = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlock) s += x[i] * x[i];
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(s / static_cast<float>(H) + 1e-6f);
    const float hs = 1.0f / static_cast<float>(H);
    for (int m = 0; m < nm; ++m) {
        float a = 0.f;
        for (int i = threadIdx.x; i < H; i += kBlock) a += router[static_cast<int64_t>(m) * H + i] * (x[i] * inv * router_norm[i] * hs);
        a = block_sum(a, red);
        if (threadIdx.x == 0) mod[m] = tanhf(a);
    }
    __syncthreads();
}

// forward_altup_predict (layers.mojo:545-581): coef[in][out] = sum_r pc[r][out][in] mod[r];
// pred[out] = streams[out] + sum_in streams[in] coef[in][out].
__global__ void __launch_bounds__(kBlock) k_altup_predict(float *pred, const float *streams, const float *router,
                                                          const float *router_norm, const float *pc, int H, int nm) {
    __shared__ float red[kBlock / 32];
    __shared__ float mod[kMaxModalities], coef[kMaxModalities * kMaxModalities];
    router_modalities(mod, streams, router, router_norm, H, nm, red);
    if (threadIdx.x < nm * nm) {
        const int in = threadIdx.x / nm, out = threadIdx.x - in * nm;
        float c = 0.f;
        for (int r = 0; r < nm; ++r) c += pc[(r * nm + out) * nm + in] * mod[r];
        coef[in * nm + out] = c;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < H; d += kBlock)
        for (int out = 0; out < nm; ++out) {
            float v = streams[static_cast<int64_t>(out) * H + d];
            for (int in = 0; in < nm; ++in) v += streams[static_cast<int64_t>(in) * H + d] * coef[in * nm + out];
            pred[static_cast<int64_t>(out) * H + d] = v;
        }
}

// forward_altup_correct (layers.mojo:584-619) fused with the output scale of the active stream
// (827-829): corr[out] = 1 + sum_r cc[r][out] mod[r]; corrected[out] = pred[out] + (act - pred[0]) corr[out];
// first = corrected[0] * output_scale.
__global__ void __launch_bounds__(kBlock) k_altup_correct(float *corrected, float *first, const float *pred,
                                                          const float *activated, const float *router,
                                                          const float *router_norm, const float *cc,
                                                          const float *out_scale, int H, int nm) {
    __shared__ float red[kBlock / 32];
    __shared__ float mod[kMaxModalities], corr[kMaxModalities];
    router_modalities(mod, activated, router, router_norm, H, nm, red);
    if (threadIdx.x < nm) {
        float c = 1.0f;
        for (int r = 0; r < nm; ++r) c += cc[r * nm + threadIdx.x] * mod[r];
        corr[threadIdx.x] = c;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < H; d += kBlock) {
        const float innov = activated[d] - pred[d];
        for (int out = 0; out < nm; ++out) {
            const int64_t i = static_cast<int64_t>(out) * H + d;
            corrected[i] = pred[i] + innov * corr[out];
        }
        first[d] = corrected[d] * out_scale[d];
    }
}

// q/k/v heads (layers.mojo:425-441): weighted norm + RoPE on q and k heads, unit norm on v heads,
// K/V rows written at pos.  One CTA per head: blocks [0, hq) q heads, [hq, hq + hkv) k and v heads.
__global__ void __launch_bounds__(kBlock) k_qkv_heads(float *q, float *k, float *v, const float *q_norm,
                                                      const float *k_norm, const float *cos_t, const float *sin_t,
                                                      const int32_t *posp, int hq, int hkv, int hd, float *kc,
                                                      float *vc) {
    __shared__ float red[kBlock / 32];
    const int pos = *posp;
    const int h = blockIdx.x;
    const bool is_q = h < hq;
    float *x = is_q ? q + static_cast<int64_t>(h) * hd : k + static_cast<int64_t>(h - hq) * hd;
    const float *nw = is_q ? q_norm : k_norm;
    float s = 0.f;
    for (int i = threadIdx.x; i < hd; i += kBlock) s += x[i] * x[i];
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(s / static_cast<float>(hd) + 1e-6f);
    const int half = hd / 2;
    const float *c = cos_t + static_cast<int64_t>(pos) * hd, *sn = sin_t + static_cast<int64_t>(pos) * hd;
    // rope_rotate (ops.mojo:33-66) on the normed head
    for (int i = threadIdx.x; i < half; i += kBlock) {
        const float x1 = x[i] * inv * nw[i], x2 = x[i + half] * inv * nw[i + half];
        const float r1 = x1 * c[i] - x2 * sn[i], r2 = x2 * c[i] + x1 * sn[i];
        if (is_q) {
            x[i] = r1;
            x[i + half] = r2;
        } else {
            const int64_t o = (static_cast<int64_t>(pos) * hkv + (h - hq)) * hd;
            kc[o + i] = r1;
            kc[o + i + half] = r2;
        }
    }
    if (!is_q) {
        const float *vh = v + static_cast<int64_t>(h - hq) * hd;
        float sv = 0.f;
        for (int i = threadIdx.x; i < hd; i += kBlock) sv += vh[i] * vh[i];
        sv = block_sum(sv, red);
        const float iv = 1.0f / sqrtf(sv / static_cast<float>(hd) + 1e-6f);
        const int64_t o = (static_cast<int64_t>(pos) * hkv + (h - hq)) * hd;
        for (int i = threadIdx.x; i < hd; i += kBlock) vc[o + i] = vh[i] * iv;
    }
}

// Attention of one q head over positions 0..pos, scaling 1.0 (layers.mojo:443-475); scores in
// dynamic shared memory (capacity floats).  Cache [cap][hkv][hd].
__global__ void __launch_bounds__(kBlock) k_attention(float *out, const float *q, const float *kc, const float *vc,
                                                      const int32_t *posp, int hq, int hkv, int hd) {
    extern __shared__ float sc[];
    __shared__ float red[kBlock / 32];
    const int pos = *posp;
    const int h = blockIdx.x, kvh = h / (hq / hkv);
    const float *qh = q + static_cast<int64_t>(h) * hd;
    float mx = -1e9f;  // softmax seeds its max at -1e9 (ops.mojo:139-182)
    for (int t = threadIdx.x; t <= pos; t += kBlock) {
        const float *kh = kc + (static_cast<int64_t>(t) * hkv + kvh) * hd;
        float s = 0.f;
        for (int d = 0; d < hd; ++d) s += qh[d] * kh[d];
        sc[t] = s;
        mx = fmaxf(mx, s);
    }
    mx = block_max(mx, red);
    float sum = 0.f;
    for (int t = threadIdx.x; t <= pos; t += kBlock) {
        const float e = expf(sc[t] - mx);
        sc[t] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    const float inv = 1.0f / sum;
    for (int d = threadIdx.x; d < hd; d += kBlock) {
        float acc = 0.f;
        for (int t = 0; t <= pos; ++t) acc += (sc[t] * inv) * vc[(static_cast<int64_t>(t) * hkv + kvh) * hd + d];
        out[static_cast<int64_t>(h) * hd + d] = acc;
    }
}

// (active + attn_norm + laurel) / sqrt(2) (layers.mojo:800-802).
__global__ void k_combine3(float *out, const float *a, const float *b, const float *c, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = (a[i] + b[i] + c[i]) * 0.7071067811865475f;
}

// _apply_nano_activation_sparsity (layers.mojo:121-147): relu(g - (mean + std * z)), z = 1.6448536.
__global__ void __launch_bounds__(kBlock) k_sparsity(float *g, int n) {
    __shared__ float red[kBlock / 32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += kBlock) s += g[i];
    const float mean = block_sum(s, red) / static_cast<float>(n);
    float v = 0.f;
    for (int i = threadIdx.x; i < n; i += kBlock) {
        const float d = g[i] - mean;
        v += d * d;
    }
    const float sd = sqrtf(block_sum(v, red) / static_cast<float>(n));
    const float cutoff = mean + sd * 1.6448536269514722f;
    for (int i = threadIdx.x; i < n; i += kBlock) g[i] = fmaxf(g[i] - cutoff, 0.f);
}

// gelu(gate) * other (geglu, ops.mojo:5-30; the per-layer gate of layers.mojo:494-498).
__global__ void k_gelu_mul(float *out, const float *gate, const float *other, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = gate[i];
        out[i] = 0.5f * x * (1.0f + erff(x / 1.4142135623730951f)) * other[i];
    }
}

// Next streams (layers.mojo:831-838): stream 0 = corrected[0]; streams m >= 1 = corrected[m] + delta.
__global__ void k_streams_next(float *streams, const float *corrected, const float *delta, int H, int nm) {
    const int64_t n = static_cast<int64_t>(nm) * H;
    for (int64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        streams[i] = corrected[i] + (i >= H ? delta[i % H] : 0.f);
}

// _collapse_altup_streams (layers.mojo:696-725): (stream0 + sum_m u_m * mag(stream0) / max(mag(u_m), 1e-6)) / nm,
// u_m = unembed_{m-1} . stream_m (given), then the final weighted norm (layers.mojo:956).  One CTA.
__global__ void __launch_bounds__(kBlock) k_collapse(float *out, const float *streams, const float *u,
                                                     const float *final_norm, int H, int nm) {
    __shared__ float red[kBlock / 32];
    __shared__ float scale[kMaxModalities];
    float s0 = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlock) s0 += streams[i] * streams[i];
    s0 = block_sum(s0, red);
    const float target = sqrtf(s0 / static_cast<float>(H) + 1e-6f);
    for (int m = 1; m < nm; ++m) {
        const float *um = u + static_cast<int64_t>(m - 1) * H;
        float s = 0.f;
        for (int i = threadIdx.x; i < H; i += kBlock) s += um[i] * um[i];
        s = block_sum(s, red);
        if (threadIdx.x == 0) scale[m] = target / fmaxf(sqrtf(s / static_cast<float>(H) + 1e-6f), 1e-6f);
    }
    __syncthreads();
    const float inv_nm = 1.0f / static_cast<float>(nm);
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlock) {
        float a = streams[i];
        for (int m = 1; m < nm; ++m) a += u[static_cast<int64_t>(m - 1) * H + i] * scale[m];
        a *= inv_nm;
        out[i] = a;
        ss += a * a;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(H) + 1e-6f);
    for (int i = threadIdx.x; i < H; i += kBlock) out[i] = out[i] * inv * final_norm[i];
}

// emb_acc += hidden (forward_nano_sequence's running sum, layers.mojo:1057-1058).
__global__ void k_accumulate(float *acc, const float *x, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) acc[i] += x[i];
}

}  // namespace nano
}  // namespace mg

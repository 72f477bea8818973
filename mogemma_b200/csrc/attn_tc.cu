// attn_tc.cu -- tensor-core attention of the batched prefill and the encoder
// (the attention of layers.mojo:63-94 for a whole packed batch of sequences):
// out = softmax(scale . Q K^T + mask) V per q head, with bf16 Q, K, V and fp32
// accumulation.
//
// Work unit: one CTA per (tile of 128 queries of one sequence, q head).  Keys
// run in blocks of 64 over the tile's key range; the mask keeps, for query
// position p of a sequence of len tokens, key positions
//   causal:  [lo(p), p]                      lo(p) = p - window + 1 on local layers, else 0
//   encoder: [lo(p), min(len - 1, p + window - 1)] on local layers, [0, len - 1] on global ones.
//
// Inputs are packed by token (the sequence's tokens contiguous, in position
// order): Q [N][Hq*hd], K [N][Hkv*hd] and V^T [Hkv*hd][N] (keys contiguous, so
// that V is a K-major operand of P.V), all bf16.
//
// Warps of a CTA (192 threads):
//  * warp 4, one lane: TMA producer -- the Q tile once, then per key block the
//    K tile (hd/64 boxes of 64 x 64) and the V^T tile (one box of 64 keys x hd)
//    into two stages;
//  * warp 5: allocates 512 TMEM columns (O: hd columns; S: two stages of 64)
//    and one lane issues tcgen05.mma: S[j&1] = Q K_j^T (M=128, N=64), then,
//    once P_j is in shared memory, O += P_j V_j (M=128, N=hd); S_{j+1} is issued
//    before P_j V_j so that it overlaps the softmax of block j;
//  * warps 0-3: softmax, one query row per thread (TMEM lane = row): S row from
//    TMEM, mask, running max, P = exp2(S - m) rounded to bf16 into a shared
//    P stage (128-byte swizzled K-major, the layout the MMA reads), row sum l
//    of the rounded P; then the epilogue O / l -> bf16.
// K, V^T, S and P are double-buffered, so block j + 1's loads and Q.K^T run
// under block j's softmax and P.V.
// The running max m is only moved when a block's max exceeds it by more than
// 8 (log2 units): P stays below 2^8 and O (in TMEM) is rescaled only on such
// a move, so most blocks need no O round trip.  O and l always share the same
// m, so the result is exact up to the bf16 rounding of P.
//
// Every mbarrier wait is bounded (common.cuh): on expiry the kernel records an
// error code, abandons the tile, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "tc_common.cuh"

namespace mg {
namespace tc {
constexpr int kAttM = 128;  // queries per tile (TMEM lanes)
constexpr int kAttBN = 64;  // keys per block (one 128-byte swizzle atom of V^T and P)
constexpr int kAttThreads = 192;
constexpr uint32_t kAttTmemCols = 512;
constexpr float kAttRescale = 8.0f;  // log2 of the largest P before the running max moves
constexpr uint32_t kErrAttQ = 0x24000000u, kErrAttK = 0x25000000u, kErrAttS = 0x26000000u,
                   kErrAttP = 0x27000000u, kErrAttV = 0x28000000u, kErrAttPV = 0x29000000u;

template <int HD>
struct AttCfg {
    static constexpr uint32_t kQBytes = kAttM * HD * 2;   // HD/64 boxes of 128 rows x 128 B
    static constexpr uint32_t kKBytes = kAttBN * HD * 2;  // per stage: HD/64 boxes of 64 keys x 128 B
    static constexpr uint32_t kVBytes = HD * kAttBN * 2;  // per stage: 1 box of 64 keys x HD rows
    static constexpr uint32_t kPBytes = kAttM * kAttBN * 2;  // per stage
    static constexpr size_t kSmem = 1024 + kQBytes + 2 * (kKBytes + kVBytes + kPBytes);
};

__device__ __forceinline__ float fast_exp2(float x) {  // PTX ex2.approx: one MUFU op, ~2 ulp
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// tiles[i] = {start (packed index of the sequence's first token), len, q0 (first query position), 0}
//
// Two stages of K, V^T, S (TMEM) and P: the loads and Q.K^T of block j + 1 run
// while the softmax of block j does.  Per stage st = j & 1 (n-th use: j >> 1):
//   k_full / v_full   TMA -> MMA                 k_empty  QK_j done -> TMA (K_{j+2})
//   s_full            QK_j done -> softmax       s_free   softmax read S_j -> MMA (QK_{j+2})
//   p_full            softmax wrote P_j -> MMA   pv_done  PV_j done -> TMA (V_{j+2}), softmax (P_{j+2},
//                                                         and O rescale before P_{j+1}), epilogue
template <int HD>
__global__ void __launch_bounds__(kAttThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v, const int4 *tiles, int gq, int window, int bidir,
                   float scale_log2, __nv_bfloat16 *out, int64_t out_ld, uint32_t *err) {
    using Cfg = AttCfg<HD>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_q, k_full[2], k_empty[2], v_full[2], s_full[2], s_free[2], p_full[2],
        pv_done[2];
    __shared__ uint32_t tmem_slot;
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023);
    const uint32_t sq = smem_u32(reinterpret_cast<void *>(base));
    const uint32_t sk = sq + Cfg::kQBytes;          // 2 K stages
    const uint32_t sv = sk + 2 * Cfg::kKBytes;      // 2 V stages
    const uint32_t sp = sv + 2 * Cfg::kVBytes;      // 2 P stages
    unsigned char *p_gen = reinterpret_cast<unsigned char *>(base) + Cfg::kQBytes + 2 * (Cfg::kKBytes + Cfg::kVBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int4 tile = tiles[blockIdx.x];
    const int start = tile.x, len = tile.y, q0 = tile.z;
    const int h = blockIdx.y, kvh = h / gq;
    // key positions the tile needs, as packed indices [kb0, kb0 + nblk * kAttBN)
    const int qlast = min(q0 + kAttM - 1, len - 1);
    const int kp_lo = window > 0 ? max(0, q0 - window + 1) : 0;
    const int kp_hi = bidir ? (window > 0 ? min(len - 1, qlast + window - 1) : len - 1) : qlast;
    const int kb0 = (start + kp_lo) & ~7;  // 16-byte aligned x for the V^T boxes
    const int nblk = (start + kp_hi + 1 - kb0 + kAttBN - 1) / kAttBN;

    if (threadIdx.x == 0) {
        mbar_init(&bar_q, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&k_full[b], 1);
            mbar_init(&k_empty[b], 1);
            mbar_init(&v_full[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&s_free[b], 4);
            mbar_init(&p_full[b], 4);
            mbar_init(&pv_done[b], 1);
        }
        fence_barrier_init();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kAttTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t t_o = tmem, t_s0 = tmem + HD;  // O: HD columns; S stages: 64 columns each

    if (warp == 4) {
        if (lane == 0) {  // TMA producer
            mbar_arrive_expect_tx(&bar_q, Cfg::kQBytes);
#pragma unroll
            for (int a = 0; a < HD / 64; ++a)
                tma_load_2d(sq + a * kAttM * 128, &map_q, h * HD + 64 * a, start + q0, smem_u32(&bar_q));
            for (int j = 0; j < nblk; ++j) {
                const int st = j & 1;
                const uint32_t use = static_cast<uint32_t>(j >> 1);  // n-th use of the stage
                const int k0 = kb0 + j * kAttBN;
                if (j >= 2 && !mbar_wait(&k_empty[st], (use - 1) & 1u, err, kErrAttK)) break;
                mbar_arrive_expect_tx(&k_full[st], Cfg::kKBytes);
#pragma unroll
                for (int a = 0; a < HD / 64; ++a)
                    tma_load_2d(sk + st * Cfg::kKBytes + a * kAttBN * 128, &map_k, kvh * HD + 64 * a, k0,
                                smem_u32(&k_full[st]));
                if (j >= 2 && !mbar_wait(&pv_done[st], (use - 1) & 1u, err, kErrAttV)) break;
                mbar_arrive_expect_tx(&v_full[st], Cfg::kVBytes);
                tma_load_2d(sv + st * Cfg::kVBytes, &map_v, k0, kvh * HD, smem_u32(&v_full[st]));
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t kIdS = idesc_bf16(kAttM, kAttBN), kIdO = idesc_bf16(kAttM, HD);
            auto issue_s = [&](int j) -> bool {
                const int st = j & 1;
                const uint32_t use = static_cast<uint32_t>(j >> 1);
                if (!mbar_wait(&k_full[st], use & 1u, err, kErrAttK)) return false;
                if (j >= 2 && !mbar_wait(&s_free[st], (use - 1) & 1u, err, kErrAttS)) return false;
                tc_fence_after();
                const uint32_t t_s = t_s0 + st * kAttBN;
                const uint32_t kbase = sk + st * Cfg::kKBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_bf16(t_s, sw128_desc(sq + (kk >> 2) * kAttM * 128 + (kk & 3) * 32),
                              sw128_desc(kbase + (kk >> 2) * kAttBN * 128 + (kk & 3) * 32), kIdS, kk > 0 ? 1u : 0u);
                umma_commit(smem_u32(&s_full[st]));
                umma_commit(smem_u32(&k_empty[st]));
                return true;
            };
            bool ok = mbar_wait(&bar_q, 0u, err, kErrAttQ) && issue_s(0);
            for (int j = 0; ok && j < nblk; ++j) {
                const int st = j & 1;
                const uint32_t use = static_cast<uint32_t>(j >> 1);
                if (j + 1 < nblk && !issue_s(j + 1)) break;
                if (!mbar_wait(&p_full[st], use & 1u, err, kErrAttP) ||
                    !mbar_wait(&v_full[st], use & 1u, err, kErrAttV))
                    break;
                tc_fence_after();
                const uint32_t pbase = sp + st * Cfg::kPBytes, vbase = sv + st * Cfg::kVBytes;
#pragma unroll
                for (int kk = 0; kk < kAttBN / 16; ++kk)
                    umma_bf16(t_o, sw128_desc(pbase + kk * 32), sw128_desc(vbase + kk * 32), kIdO,
                              (j | kk) != 0 ? 1u : 0u);
                umma_commit(smem_u32(&pv_done[st]));
            }
        }
    } else {  // softmax warps: thread = query row r of the tile
        const int r = warp * 32 + lane;
        const int qp = q0 + r;
        const bool qvalid = qp < len;
        const int lo = window > 0 ? max(0, qp - window + 1) : 0;
        const int hi = !qvalid ? -1 : (bidir ? (window > 0 ? min(len - 1, qp + window - 1) : len - 1) : qp);
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            const int st = j & 1;
            const uint32_t use = static_cast<uint32_t>(j >> 1);
            ok = mbar_wait(&s_full[st], use & 1u, err, kErrAttS);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // pass 1: masked, scaled block max (S is read from TMEM again in pass 2)
            const uint32_t t_s = t_s0 + st * kAttBN + lane_off;
            const int kpos0 = kb0 + j * kAttBN - start;
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < kAttBN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(t_s + 32 * c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int kp = kpos0 + 32 * c + i;
                    if (kp >= lo && kp <= hi) mx = fmaxf(mx, __uint_as_float(v[i]) * scale_log2);
                }
            }
            const float m_new = mx > m_ref + kAttRescale ? mx : m_ref;
            const float alpha = m_new == m_ref ? 1.f : fast_exp2(m_ref - m_new);
            // O must hold P_{j-1} V_{j-1} before it is rescaled for block j
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                const int pj = j - 1;
                ok = mbar_wait(&pv_done[pj & 1], static_cast<uint32_t>(pj >> 1) & 1u, err, kErrAttPV);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(t_o + lane_off + 32 * c, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(t_o + lane_off + 32 * c, o);
                }
            }
            // P stage st is free once P_{j-2} V_{j-2} has completed
            if (j >= 2) {
                ok = mbar_wait(&pv_done[st], (use - 1) & 1u, err, kErrAttPV);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
            }
            // pass 2: P = exp2(S - m) as bf16 into the swizzled P stage, row sum of the rounded values
            float sum = 0.f;
            unsigned char *prow = p_gen + st * Cfg::kPBytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll 1
            for (int c = 0; c < kAttBN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(t_s + 32 * c, v);
#pragma unroll
                for (int g = 0; g < 4; ++g) {  // 8 keys = one 16-byte chunk
                    uint32_t pk[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int i0 = 8 * g + 2 * i;
                        const int kp = kpos0 + 32 * c + i0;
                        const bool v0 = m_new != -INFINITY && kp >= lo && kp <= hi;
                        const bool v1 = m_new != -INFINITY && kp + 1 >= lo && kp + 1 <= hi;
                        const float a = v0 ? fast_exp2(__uint_as_float(v[i0]) * scale_log2 - m_new) : 0.f;
                        const float b = v1 ? fast_exp2(__uint_as_float(v[i0 + 1]) * scale_log2 - m_new) : 0.f;
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(a, b);
                        sum += __low2float(pr) + __high2float(pr);
                        pk[i] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    const int chunk = 4 * c + g;  // 16-byte chunk of the 128-byte row
                    *reinterpret_cast<uint4 *>(prow + ((chunk ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            }
            l = l * alpha + sum;
            m_ref = m_new;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_free[st]);
                mbar_arrive(&p_full[st]);
            }
        }
        if (ok) {
            const int lj = nblk - 1;
            ok = mbar_wait(&pv_done[lj & 1], static_cast<uint32_t>(lj >> 1) & 1u, err, kErrAttPV);
        }
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            const float inv_l = l > 0.f ? 1.0f / l : 0.f;
            __nv_bfloat16 *dst = out + static_cast<int64_t>(start + qp) * out_ld + static_cast<int64_t>(h) * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(t_o + lane_off + 32 * c, o);
                if (qvalid) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(__uint_as_float(o[2 * i]) * inv_l,
                                                                        __uint_as_float(o[2 * i + 1]) * inv_l);
                        pk[i] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst + 32 * c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAttTmemCols));
}

template <int HD>
static cudaError_t launch_attn_tc(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                                  const int4 *tiles, int ntiles, int Hq, int gq, int window, int bidir,
                                  float scale_log2, __nv_bfloat16 *out, int64_t out_ld, uint32_t *err,
                                  cudaStream_t s) {
    static bool attr = false;
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(AttCfg<HD>::kSmem));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    attn_tc_kernel<HD><<<dim3(ntiles, Hq), kAttThreads, AttCfg<HD>::kSmem, s>>>(mq, mk, mv, tiles, gq, window, bidir,
                                                                                scale_log2, out, out_ld, err);
    return cudaGetLastError();
}
}  // namespace tc

// Head dims the tensor-core attention handles.
bool attn_tc_supported(int hd) { return hd == 64 || hd == 128 || hd == 256; }

// qb [N][Hq*hd], kb [N][Hkv*hd], vt [Hkv*hd][vt_ld] (vt_ld a multiple of 8,
// columns >= N unread), all bf16; out [N][out_ld] bf16 (head h at column h*hd;
// out_ld a multiple of 8).  window: the local window (0 on global layers);
// bidir: encoder mask instead of the causal one.
cudaError_t attn_tc(const __nv_bfloat16 *qb, const __nv_bfloat16 *kb, const __nv_bfloat16 *vt, int64_t vt_ld, int N,
                    int Hq, int Hkv, int hd, const int4 *tiles, int ntiles, int window, int bidir, float scale,
                    __nv_bfloat16 *out, int64_t out_ld, uint32_t *err, cudaStream_t s) {
    using namespace tc;
    if (!attn_tc_supported(hd) || Hq % Hkv != 0 || vt_ld % 8 != 0 || out_ld % 8 != 0) return cudaErrorInvalidValue;
    if (ntiles == 0) return cudaSuccess;
    CUtensorMap mq, mk, mv;
    if (!make_map_bf16(&mq, qb, N, static_cast<int64_t>(Hq) * hd, static_cast<int64_t>(Hq) * hd, kAttM) ||
        !make_map_bf16(&mk, kb, N, static_cast<int64_t>(Hkv) * hd, static_cast<int64_t>(Hkv) * hd, kAttBN) ||
        !make_map_bf16(&mv, vt, static_cast<int64_t>(Hkv) * hd, N, vt_ld, hd))
        return cudaErrorInvalidValue;
    const float scale_log2 = scale * 1.4426950408889634f;
    if (hd == 256)
        return launch_attn_tc<256>(mq, mk, mv, tiles, ntiles, Hq, Hq / Hkv, window, bidir, scale_log2, out, out_ld,
                                   err, s);
    if (hd == 128)
        return launch_attn_tc<128>(mq, mk, mv, tiles, ntiles, Hq, Hq / Hkv, window, bidir, scale_log2, out, out_ld,
                                   err, s);
    return launch_attn_tc<64>(mq, mk, mv, tiles, ntiles, Hq, Hq / Hkv, window, bidir, scale_log2, out, out_ld, err,
                              s);
}

}  // namespace mg

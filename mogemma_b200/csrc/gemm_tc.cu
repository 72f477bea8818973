// gemm_tc.cu -- tcgen05 tensor-core GEMM, the dense contraction of the batched
// (prefill) path: C[M][N] (fp32) = A[M][K] (bf16) . B[N][K]^T (bf16), both
// operands K-major (activations [tokens][features], weights [out][in] as the
// reference stores them, convert.py:92-121).
//
// One CTA computes a 128 x 128 tile of C with 4 warps:
//  * warp 0, one lane: TMA producer -- 2-D tiled bulk tensor loads of a
//    128 x 64 A tile and a 128 x 64 B tile per stage (128-byte swizzle) into a
//    4-stage ring, completing on the stage's mbarrier;
//  * warp 1: allocates 128 TMEM columns (the fp32 accumulator, 128 lanes x 128
//    columns); one lane issues tcgen05.mma (M=128, N=128, K=16, bf16 -> f32) four
//    times per stage from shared-memory descriptors, and tcgen05.commit releases
//    the stage once the MMAs have read it;
//  * all 4 warps: epilogue -- warp w reads TMEM lanes 32w..32w+31 (rows of the
//    tile) with tcgen05.ld and stores them to C.
// Every mbarrier wait is bounded (common.cuh); on expiry the kernel records an
// error code, skips the rest of the work, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/mogemma_b200.h"
#include "common.cuh"
#include "tc_common.cuh"

namespace mg {
mg_status report_error(mg_status st, const char *msg);

namespace tc {
constexpr int kBM = 128;   // tile rows (TMEM lanes)
constexpr int kBN = 128;   // tile columns (TMEM columns)
constexpr int kBK = 64;    // K per stage: 64 bf16 = 128 bytes, one swizzle row
constexpr int kUK = 16;    // K of one tcgen05.mma (kind::f16)
constexpr int kStages = 3;  // 97 KB of shared memory: two CTAs per SM, one's epilogue under the other's MMAs
constexpr int kThreads = 128;
constexpr uint32_t kABytes = kBM * kBK * 2;
constexpr uint32_t kBBytes = kBN * kBK * 2;
constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * (kABytes + kBBytes);
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kErrTcFull = 0x21000000u, kErrTcEmpty = 0x22000000u, kErrTcDone = 0x23000000u;

constexpr uint32_t kIdesc = idesc_bf16(kBM, kBN);

// Split-K: blockIdx.z takes k steps [z nk_split, (z + 1) nk_split) and writes
// its partial product to C + z c_split (a workspace the caller reduces).
__global__ void __launch_bounds__(kThreads, 2)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        float *C, int M, int N, int K, int64_t ldc, int nk_split, int64_t c_split, uint32_t *err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kStages], empty[kStages], done;
    __shared__ uint32_t tmem_slot;
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023);
    const uint32_t sa = smem_u32(reinterpret_cast<void *>(base));
    const uint32_t sb = sa + kStages * kABytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int kbeg = blockIdx.z * nk_split;
    const int nk = min(nk_split, K / kBK - kbeg);  // k steps of this split (>= 1)
    C += blockIdx.z * c_split;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0 && lane == 0) {
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kStages;
            if (kt >= kStages && !mbar_wait(&empty[s], ((kt / kStages) - 1) & 1u, err, kErrTcEmpty)) break;
            mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
            tma_load_2d(sa + s * kABytes, &map_a, (kbeg + kt) * kBK, m0, smem_u32(&full[s]));
            tma_load_2d(sb + s * kBBytes, &map_b, (kbeg + kt) * kBK, n0, smem_u32(&full[s]));
        }
    } else if (warp == 1 && lane == 0) {
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kStages;
            if (!mbar_wait(&full[s], (kt / kStages) & 1u, err, kErrTcFull)) break;
            tc_fence_after();
            const uint32_t a0 = sa + s * kABytes, b0 = sb + s * kBBytes;
#pragma unroll
            for (int k = 0; k < kBK / kUK; ++k)
                umma_bf16(tmem, sw128_desc(a0 + k * kUK * 2), sw128_desc(b0 + k * kUK * 2), kIdesc, (kt | k) != 0 ? 1u : 0u);
            umma_commit(smem_u32(&empty[s]));
        }
        umma_commit(smem_u32(&done));  // arrives once every MMA issued above has completed
    }
    __syncwarp();

    // epilogue: warp w owns TMEM lanes (tile rows) 32w .. 32w + 31.  Each 32 x 32
    // block goes through shared memory (the ring is free once `done` fired; a
    // padded [32][33] float tile per warp) so that every global store of the
    // warp writes 32 consecutive floats of one row.
    const bool have = mbar_wait(&done, 0u, err, kErrTcDone);
    tc_fence_after();
    // tcgen05.ld is warp-collective: decide per warp
    if (__all_sync(0xffffffffu, have && ld_relaxed_u32(err) == 0u)) {
        float *stage = reinterpret_cast<float *>(base) + warp * 32 * 33;
        const int row0 = m0 + warp * 32;
        for (int c0 = 0; c0 < kBN; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c0), v);
#pragma unroll
            for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = __uint_as_float(v[j]);
            __syncwarp();
            const int col = n0 + c0 + lane;
            if (col < N) {
                const int rows = min(32, M - row0);
#pragma unroll 4
                for (int rr = 0; rr < rows; ++rr) C[static_cast<int64_t>(row0 + rr) * ldc + col] = stage[rr * 33 + lane];
            }
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace tc

namespace tc {
// ---- persistent variant for grids with at least one 128 x 256 tile per SM:
// one CTA per SM walks the tiles.
//  * warp 0, one lane: TMA producer over a 4-stage ring (128 x 64 A + 256 x 64 B per stage);
//  * warp 1: allocates 512 TMEM columns = two 256-column fp32 accumulators; one
//    lane issues tcgen05.mma (M=128, N=256, K=16) into the free accumulator and
//    commits it to acc_full when the tile's K loop is issued;
//  * warps 2-5: epilogue of the other accumulator (warp w reads TMEM lanes
//    32 (w % 4) ..), staged through a padded [32][33] float tile per warp so
//    every store of a warp writes 32 consecutive floats of one row; then the
//    accumulator is handed back (acc_empty).
// So a tile's epilogue runs under the next tile's MMAs.
// GEGLU: B holds gate and up rows in alternating blocks of 128 (rows
// 256 j .. 256 j + 127 gate features 128 j .., the next 128 the up rows of the
// same features), so each tile has both halves of 128 features and the
// epilogue writes act[m][128 j + c] = bf16(gelu_erf(gate) * up) (ops.mojo:5-30)
// instead of the fp32 products.
constexpr int kPBN = 256;
constexpr int kPStages = 4;
constexpr int kPThreads = 192;
constexpr uint32_t kPABytes = kBM * kBK * 2;
constexpr uint32_t kPBBytes = kPBN * kBK * 2;
constexpr size_t kPSmem = 1024 + static_cast<size_t>(kPStages) * (kPABytes + kPBBytes) + 4 * 32 * 33 * 4;
constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPIdesc = idesc_bf16(kBM, kPBN);
constexpr uint32_t kErrTcAcc = 0x2A000000u;

template <bool GEGLU>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_bf16_tc_persistent_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                                   float *C, __nv_bfloat16 *act, int M, int N, int K, int64_t ldc, uint32_t *err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kPStages], empty[kPStages], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023);
    const uint32_t sa = smem_u32(reinterpret_cast<void *>(base));
    const uint32_t sb = sa + kPStages * kPABytes;
    float *stage_all = reinterpret_cast<float *>(base + kPStages * (kPABytes + kPBBytes));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + kPBN - 1) / kPBN;
    const int ntiles = ((M + kBM - 1) / kBM) * tiles_n;
    const int nk = K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kPTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kPBN;
                for (int kt = 0; kt < nk; ++kt, ++it) {
                    const uint32_t s = it % kPStages;
                    if (it >= kPStages && !mbar_wait(&empty[s], ((it / kPStages) - 1) & 1u, err, kErrTcEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kPABytes + kPBBytes);
                    tma_load_2d(sa + s * kPABytes, &map_a, kt * kBK, m0, smem_u32(&full[s]));
                    tma_load_2d(sb + s * kPBBytes, &map_b, kt * kBK, n0, smem_u32(&full[s]));
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0, i = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++i) {
                const uint32_t b = i & 1u;
                if (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1u, err, kErrTcAcc)) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * kPBN;
                for (int kt = 0; kt < nk; ++kt, ++it) {
                    const uint32_t s = it % kPStages;
                    if (!mbar_wait(&full[s], (it / kPStages) & 1u, err, kErrTcFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sa + s * kPABytes, b0 = sb + s * kPBBytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUK; ++k)
                        umma_bf16(acc, sw128_desc(a0 + k * kUK * 2), sw128_desc(b0 + k * kUK * 2), kPIdesc,
                                  (kt | k) != 0 ? 1u : 0u);
                    umma_commit(smem_u32(&empty[s]));
                }
                if (ok) umma_commit(smem_u32(&acc_full[b]));
            }
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may read
        float *stage = stage_all + (warp - 2) * 32 * 33;
        uint32_t i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            const uint32_t b = i & 1u;
            const bool ok = mbar_wait(&acc_full[b], (i >> 1) & 1u, err, kErrTcDone);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kPBN;
            const int row0 = m0 + q * 32;
            const int rows = min(32, M - row0);
            const uint32_t t_acc = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * kPBN;
            if constexpr (GEGLU) {
                for (int c0 = 0; c0 < kPBN / 2; c0 += 32) {
                    uint32_t g[32], u[32];
                    tmem_ld32(t_acc + static_cast<uint32_t>(c0), g);
                    tmem_ld32(t_acc + static_cast<uint32_t>(kPBN / 2 + c0), u);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float gv = __uint_as_float(g[j]);
                        stage[lane * 33 + j] = 0.5f * gv * (1.0f + erff(gv * kInvSqrt2)) * __uint_as_float(u[j]);
                    }
                    __syncwarp();
                    const int f = n0 / 2 + c0 + lane;
                    if (f < N / 2) {
#pragma unroll 4
                        for (int rr = 0; rr < rows; ++rr)
                            act[static_cast<int64_t>(row0 + rr) * ldc + f] = __float2bfloat16_rn(stage[rr * 33 + lane]);
                    }
                    __syncwarp();
                }
            } else {
                for (int c0 = 0; c0 < kPBN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(t_acc + static_cast<uint32_t>(c0), v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = __uint_as_float(v[j]);
                    __syncwarp();
                    const int col = n0 + c0 + lane;
                    if (col < N) {
#pragma unroll 4
                        for (int rr = 0; rr < rows; ++rr)
                            C[static_cast<int64_t>(row0 + rr) * ldc + col] = stage[rr * 33 + lane];
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPTmemCols));
}
}  // namespace tc

namespace tc {
// C[m][n] = sum over the splits of ws[z][m][n] (ws rows N apart, splits M N apart)
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float *ws, int splits, int M, int N, float *C,
                                                           int64_t ldc) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (i >= static_cast<int64_t>(M) * N) return;
    const int64_t m = i / N, n = i - m * N;
    float acc = 0.f;
    for (int z = 0; z < splits; ++z) acc += ws[static_cast<int64_t>(z) * M * N + i];
    C[m * ldc + n] = acc;
}

static int g_sms = 0;  // SM count of the device, set with the kernels' shared-memory limits

static cudaError_t gemm_setup() {
    if (g_sms != 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_bf16_tc_persistent_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kPSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_bf16_tc_persistent_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kPSmem));
    int dev = 0, sms = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) g_sms = sms;
    return e;
}
}  // namespace tc

// C[M][N] = A[M][K] . B[N][K]^T; A, B bf16 device memory (16-byte aligned rows),
// K a multiple of 64, err a device word that receives a code on a timeout.
// ws (optional, ws_floats long): workspace for split-K when the grid of
// 128 x 128 tiles covers under half the SMs (few output columns, e.g. the
// o_proj / down_proj of a batched decode step); the K steps are split so
// the grid fills the GPU and a reduce kernel sums the partial products.
cudaError_t gemm_bf16_tc(const void *A, int64_t lda, const void *B, int64_t ldb, float *C, int64_t ldc, int M, int N,
                         int K, uint32_t *err, cudaStream_t stream, float *ws, size_t ws_floats) {
    using namespace tc;
    const cudaError_t e = gemm_setup();
    if (e != cudaSuccess) return e;
    CUtensorMap ma, mb;
    const int ntiles = ((M + kBM - 1) / kBM) * ((N + kPBN - 1) / kPBN);
    if (ntiles >= g_sms) {  // enough 128 x 256 tiles to fill every SM: the persistent kernel
        if (!make_map_bf16(&ma, A, M, K, lda, kBM) || !make_map_bf16(&mb, B, N, K, ldb, kPBN))
            return cudaErrorInvalidValue;
        gemm_bf16_tc_persistent_kernel<false><<<std::min(ntiles, g_sms), kPThreads, kPSmem, stream>>>(
            ma, mb, C, nullptr, M, N, K, ldc, err);
        return cudaGetLastError();
    }
    if (!make_map_bf16(&ma, A, M, K, lda, kBM) || !make_map_bf16(&mb, B, N, K, ldb, kBN)) return cudaErrorInvalidValue;
    const int nk = K / kBK;
    const int tiles = ((N + kBN - 1) / kBN) * ((M + kBM - 1) / kBM);
    int splits = 1;
    if (ws && 2 * tiles < g_sms && nk >= 8) {
        splits = std::min(std::min(nk / 4, 2 * g_sms / tiles), 32);  // >= 4 k steps per split
        while (splits > 1 && static_cast<size_t>(splits) * M * N > ws_floats) --splits;
    }
    if (splits > 1) {
        const int nk_split = (nk + splits - 1) / splits;
        splits = (nk + nk_split - 1) / nk_split;  // every split non-empty
        const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM, splits);
        gemm_bf16_tc_kernel<<<grid, kThreads, kSmem, stream>>>(ma, mb, ws, M, N, K, N, nk_split,
                                                               static_cast<int64_t>(M) * N, err);
        const int64_t total = static_cast<int64_t>(M) * N;
        splitk_reduce_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(ws, splits, M, N, C,
                                                                                             ldc);
        return cudaGetLastError();
    }
    const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
    gemm_bf16_tc_kernel<<<grid, kThreads, kSmem, stream>>>(ma, mb, C, M, N, K, ldc, nk, 0, err);
    return cudaGetLastError();
}

// act[M][N2/2] (bf16, row stride ld_act) = GeGLU of A . B^T with B's rows in
// alternating 128-row gate / up blocks (N2 a multiple of 256).  Returns
// cudaErrorNotSupported, launching nothing, when the grid has fewer tiles
// than SMs; the caller then takes the fp32 product and a separate GeGLU.
cudaError_t gemm_bf16_tc_geglu(const void *A, int64_t lda, const void *B, int64_t ldb, __nv_bfloat16 *act,
                               int64_t ld_act, int M, int N2, int K, uint32_t *err, cudaStream_t stream) {
    using namespace tc;
    const cudaError_t e = gemm_setup();
    if (e != cudaSuccess) return e;
    const int ntiles = ((M + kBM - 1) / kBM) * (N2 / kPBN);
    if (N2 % kPBN != 0 || ntiles < g_sms) return cudaErrorNotSupported;
    CUtensorMap ma, mb;
    if (!make_map_bf16(&ma, A, M, K, lda, kBM) || !make_map_bf16(&mb, B, N2, K, ldb, kPBN))
        return cudaErrorInvalidValue;
    gemm_bf16_tc_persistent_kernel<true><<<std::min(ntiles, g_sms), kPThreads, kPSmem, stream>>>(
        ma, mb, nullptr, act, M, N2, K, ld_act, err);
    return cudaGetLastError();
}

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_gemm_bf16(const void *a_dev, int64_t lda, const void *b_dev, int64_t ldb, float *c_dev,
                                  int64_t ldc, int32_t M, int32_t N, int32_t K, uint32_t *err_dev, void *stream) {
    if (!a_dev || !b_dev || !c_dev || !err_dev) return report_error(MG_ERR_INVALID, "mg_gemm_bf16: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || K % tc::kBK != 0)
        return report_error(MG_ERR_INVALID, "mg_gemm_bf16: need M, N > 0 and K a positive multiple of 64");
    if (lda < K || ldb < K || ldc < N || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(a_dev) % 16 != 0 || reinterpret_cast<uintptr_t>(b_dev) % 16 != 0)
        return report_error(MG_ERR_INVALID, "mg_gemm_bf16: rows must be 16-byte aligned and strides >= extents");
    const cudaError_t e = gemm_bf16_tc(a_dev, lda, b_dev, ldb, c_dev, ldc, M, N, K, err_dev,
                                       static_cast<cudaStream_t>(stream), nullptr, 0);
    if (e != cudaSuccess) {
        char buf[160];
        snprintf(buf, sizeof buf, "mg_gemm_bf16: %s", cudaGetErrorString(e));
        return report_error(MG_ERR_CUDA, buf);
    }
    return MG_OK;
}

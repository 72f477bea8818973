// static_sample.cu -- mg_sample_static: the token draw of _sample_next_token
// (src/py/mogemma/model.py:103-150) over logits that already sit in device
// memory, using no device memory of its own beyond a fixed static array.
//
// Who calls this: a serving engine that computes the logits itself and only
// wants the draw.  Such an engine usually owns every byte of HBM through its own
// pool, reserved at start-up, and forbids allocation in its steady state:
// cudaMalloc and cudaFree synchronise the whole device (stalling every stream of
// the engine) and would take memory the pool has already promised to KV caches.
// mg_sample cannot serve it (it copies host logits into buffers it allocates);
// this entry point allocates nothing.
//
// It is a variant of the decode kernel's last two phases (per-CTA top-k of the
// lm_head rows into candidate keys, then the merge and the draw): the logits of
// each row are cut into up to 148 slices, one CTA selects the best K keys of its
// slice into a candidate array, and one CTA per row merges the candidates and
// draws.  The candidate array -- the only scratch -- is the file-scope array
// below.  Greedy (temperature <= 0) and 0 < top_k <= 64 are covered (top_p on
// top of either); the result equals mg_sample's token for token.
//
// Set-up: every call, with the calling thread's current device, looks up the
// array's device address with cudaGetSymbolAddress and raises the merge
// kernel's dynamic shared-memory limit (host-side table lookups, no
// allocation).  Nothing is cached across calls, so a context that the caller
// tears down and recreates (cudaDeviceReset) gets the new module's address.
// The first call on a device loads the library's kernels onto it; make that
// first call before any stream capture.
//
// Sharing: every call on a device uses the same array.  Two calls whose
// kernels overlap on the GPU (different streams, no ordering between them)
// race on it and may return wrong tokens; calls on one stream are ordered and
// safe.  Nothing in the array has to start at zero: every candidate slot a call
// reads was written by the same call's first kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>

#include "../../include/mogemma_b200.h"
#include "common.cuh"
#include "decode.cuh"
#include "select.cuh"

namespace mg {
mg_status report_error(mg_status st, const char *msg);

constexpr int kStThreads = 256;
constexpr int kStMaxRows = MG_SAMPLE_STATIC_MAX_ROWS;
constexpr int kStMaxSlices = MG_SAMPLE_STATIC_MAX_SLICES;
constexpr int kStSliceMin = 1024;  // vocabulary entries per slice before another slice is opened
constexpr size_t kStKeys = static_cast<size_t>(kStMaxRows) * kStMaxSlices * kMaxTopK;
constexpr size_t kStMergeSmem = static_cast<size_t>(kStMaxSlices) * kMaxTopK * sizeof(uint64_t);

// Candidate keys [row][slice][K] of the current call: 8 * 148 * 64 * 8 bytes = 606,208 bytes.
static __device__ __align__(256) uint64_t g_st_cand[kStKeys];

// One CTA per (slice, row): the K best keys of the slice, sorted, to cand.
__global__ void __launch_bounds__(kStThreads)
    st_slice_topk_kernel(const float *logits, int64_t ld, int V, int slices, int K, uint64_t *cand) {
    __shared__ SelectSmem sel;
    __shared__ uint64_t outk[kMaxTopK];
    const int s = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int per = (V + slices - 1) / slices;
    const int lo = s * per;
    const int n = max(0, min(V - lo, per));
    const float *row = logits + static_cast<int64_t>(b) * ld;
    block_select_topk(
        n, K, [&](int i) { return topk_key(__ldg(row + lo + i), static_cast<uint32_t>(lo + i)); }, outk, sel, tid,
        kStThreads, [] { __syncthreads(); });
    uint64_t *dst = cand + (static_cast<int64_t>(b) * slices + s) * K;
    for (int j = tid; j < K; j += kStThreads) dst[j] = outk[j];
}

// One CTA per row: merge slices * K candidates into the K best, then draw.
__global__ void __launch_bounds__(kStThreads)
    st_draw_kernel(const uint64_t *cand, int slices, int K, double temperature, double top_p,
                   const double *uniforms, uint64_t seed, uint64_t offset, int32_t *out) {
    extern __shared__ __align__(16) uint64_t keys[];  // [slices * K]
    __shared__ SelectSmem sel;
    __shared__ uint64_t outk[kMaxTopK];
    __shared__ double f[kMaxTopK];
    __shared__ int order[kMaxTopK];
    const int b = blockIdx.x, tid = threadIdx.x;
    const int n = slices * K;
    const uint64_t *src = cand + static_cast<int64_t>(b) * n;
    for (int i = tid; i < n; i += kStThreads) keys[i] = src[i];
    __syncthreads();
    block_select_topk(
        n, K, [&](int i) { return keys[i]; }, outk, sel, tid, kStThreads, [] { __syncthreads(); });
    if (tid == 0) {
        const double u = uniforms ? uniforms[b] : philox_uniform(seed, offset, static_cast<uint32_t>(b));
        out[b] = draw_from_sorted(outk, K, temperature, top_p, u, f, order);
    }
}

namespace {
mg_status st_error(mg_status st, const char *what, cudaError_t e) {
    char buf[256];
    snprintf(buf, sizeof buf, "mg_sample_static: %s failed: %s", what, cudaGetErrorString(e));
    return report_error(st, buf);
}

// The array's address on the current device, and the merge kernel's shared
// memory limit; repeated on every call (see the header comment).
mg_status st_setup(uint64_t **cand) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_st_cand);
    if (e != cudaSuccess) return st_error(MG_ERR_CUDA, "cudaGetSymbolAddress", e);
    e = cudaFuncSetAttribute(st_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kStMergeSmem));
    if (e != cudaSuccess) return st_error(MG_ERR_CUDA, "cudaFuncSetAttribute", e);
    *cand = static_cast<uint64_t *>(ptr);
    return MG_OK;
}
}  // namespace
}  // namespace mg

using namespace mg;

extern "C" mg_status mg_sample_static(const float *logits_dev, int64_t ld, int32_t batch, int32_t vocab,
                                      double temperature, int32_t top_k, double top_p, const double *uniforms_dev,
                                      uint64_t seed, uint64_t offset, int32_t *out_dev, void *stream) {
    char buf[256];
    if (!logits_dev || !out_dev) return report_error(MG_ERR_INVALID, "mg_sample_static: null logits or output pointer");
    if (reinterpret_cast<uintptr_t>(logits_dev) % sizeof(float) != 0)
        return report_error(MG_ERR_INVALID, "mg_sample_static: logits pointer is not 4-byte aligned");
    if (vocab <= 0 || ld < vocab) return report_error(MG_ERR_INVALID, "mg_sample_static: need vocab > 0 and ld >= vocab");
    if (batch <= 0 || batch > kStMaxRows) {
        snprintf(buf, sizeof buf, "mg_sample_static: batch %d outside 1..%d (the static candidate array holds %d rows)",
                 batch, kStMaxRows, kStMaxRows);
        return report_error(MG_ERR_INVALID, buf);
    }
    const int K = temperature <= 0.0 ? 1 : ((top_k > 0 && top_k < vocab) ? top_k : vocab);
    if (K > kMaxTopK) {
        snprintf(buf, sizeof buf,
                 "mg_sample_static: %d candidates per row exceed %d (needs temperature <= 0 or 0 < top_k <= %d)", K,
                 kMaxTopK, kMaxTopK);
        return report_error(MG_ERR_UNSUPPORTED, buf);
    }
    uint64_t *cand = nullptr;
    mg_status st = st_setup(&cand);
    if (st != MG_OK) return st;
    const int slices = std::min(kStMaxSlices, (vocab + kStSliceMin - 1) / kStSliceMin);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st_slice_topk_kernel<<<dim3(slices, batch), kStThreads, 0, s>>>(logits_dev, ld, vocab, slices, K, cand);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return st_error(MG_ERR_CUDA, "slice top-k launch", e);
    const size_t smem = static_cast<size_t>(slices) * K * sizeof(uint64_t);
    st_draw_kernel<<<batch, kStThreads, smem, s>>>(cand, slices, K, temperature, top_p, uniforms_dev, seed, offset,
                                                    out_dev);
    e = cudaGetLastError();
    if (e != cudaSuccess) return st_error(MG_ERR_CUDA, "merge/draw launch", e);
    return MG_OK;
}

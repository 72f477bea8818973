// convert.cu -- weight upload helper: converts rows of F32/BF16 host data
// (already copied to a device staging buffer) into the device layout: element
// type F32 or BF16 (round to nearest even), row stride dst_ld, zero padding.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mogemma_b200.h"
#include "select.cuh"  // philox4x32_10

namespace mg {

// Synthetic weights: rows [row0, row0 + rows) x columns [col0, col0 + cols) of a
// tensor with full_cols columns, as F32 into dst ([rows][cols]).  Element e of
// the tensor is std * N(0, 1) from Box-Muller on one Philox4x32-10 draw keyed
// by (key, e): the same values for any view of the tensor.
__global__ void synth_fill_kernel(float *dst, int64_t rows, int64_t cols, int64_t row0, int64_t col0,
                                  int64_t full_cols, uint64_t key, float std) {
    const int64_t total = rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        const uint64_t e = static_cast<uint64_t>((row0 + r) * full_cols + col0 + c);
        uint32_t ctr[4] = {static_cast<uint32_t>(e), static_cast<uint32_t>(e >> 32), 0x5eed5eedu, 0x0u};
        philox4x32_10(ctr, static_cast<uint32_t>(key), static_cast<uint32_t>(key >> 32));
        const float u1 = (static_cast<float>(ctr[0] >> 8) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
        const float u2 = static_cast<float>(ctr[1] >> 8) * (1.0f / 16777216.0f);
        dst[i] = std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}

cudaError_t synth_fill_launch(float *dst, int64_t rows, int64_t cols, int64_t row0, int64_t col0, int64_t full_cols,
                              uint64_t key, float std, cudaStream_t stream) {
    const int64_t total = rows * cols;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    synth_fill_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(dst, rows, cols, row0, col0, full_cols, key,
                                                                        std);
    return cudaGetLastError();
}

__global__ void convert_rows_kernel(const void *src, int src_dtype, int64_t rows, int64_t cols, void *dst,
                                    int dst_dtype, int64_t dst_ld) {
    const int64_t total = rows * dst_ld;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / dst_ld, c = i - r * dst_ld;
        float v = 0.f;
        if (c < cols) {
            const int64_t si = r * cols + c;
            v = src_dtype == MG_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(src)[si])
                                     : static_cast<const float *>(src)[si];
        }
        if (dst_dtype == MG_BF16)
            static_cast<__nv_bfloat16 *>(dst)[i] = __float2bfloat16_rn(v);
        else
            static_cast<float *>(dst)[i] = v;
    }
}

cudaError_t convert_rows_launch(const void *src, int src_dtype, int64_t rows, int64_t cols, void *dst, int dst_dtype,
                                int64_t dst_ld, cudaStream_t stream) {
    const int64_t total = rows * dst_ld;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    convert_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, src_dtype, rows, cols, dst, dst_dtype,
                                                                         dst_ld);
    return cudaGetLastError();
}

}  // namespace mg

namespace mg {

// Scatter rows [row_off, row_off + rows) of a [*, cols] F32/BF16 matrix (staged
// on the device) into the tiled layout [group][segment][mult*rps][kc]; `part`
// selects the row block inside a tile (0: first/only matrix, 1: up_proj rows).
__global__ void tile_rows_kernel(const void *src, int src_dtype, int64_t rows, int64_t cols, int64_t row_off,
                                 void *dst, int dst_dtype, int Kp, int rps, int mult, int kc, int nseg, int part) {
    const int64_t total = rows * Kp;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / Kp;
        const int c = static_cast<int>(i - r * Kp);
        float v = 0.f;
        if (c < cols) {
            const int64_t si = r * cols + c;
            v = src_dtype == MG_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(src)[si])
                                     : static_cast<const float *>(src)[si];
        }
        const int64_t R = row_off + r;
        const int64_t g = R / rps;
        const int j = static_cast<int>(R - g * rps);
        const int s = c / kc, cc = c - s * kc;
        const int64_t di = ((g * nseg + s) * mult * rps + static_cast<int64_t>(part) * rps + j) * kc + cc;
        if (dst_dtype == MG_BF16)
            static_cast<__nv_bfloat16 *>(dst)[di] = __float2bfloat16_rn(v);
        else
            static_cast<float *>(dst)[di] = v;
    }
}

cudaError_t tile_rows_launch(const void *src, int src_dtype, int64_t rows, int64_t cols, int64_t row_off, void *dst,
                             int dst_dtype, int Kp, int rps, int mult, int kc, int nseg, int part,
                             cudaStream_t stream) {
    const int64_t total = rows * Kp;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    tile_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, src_dtype, rows, cols, row_off, dst,
                                                                       dst_dtype, Kp, rps, mult, kc, nseg, part);
    return cudaGetLastError();
}

}  // namespace mg

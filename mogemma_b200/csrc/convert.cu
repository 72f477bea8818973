// convert.cu -- weight upload helper: converts rows of F32/BF16 host data
// (already copied to a device staging buffer) into the device layout: element
// type F32 or BF16 (round to nearest even), row stride dst_ld, zero padding.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mogemma_b200.h"

namespace mg {

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

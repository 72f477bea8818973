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

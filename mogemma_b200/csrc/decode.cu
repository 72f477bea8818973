// decode.cu -- host launch helpers of the persistent decode kernel.
//
// The kernel (decode_kernel.cuh) is instantiated once per batch row count
// (1..kMaxRows) and weight type, each row count in its own translation unit
// (decode_nb<N>.cu).  These helpers pick the instantiation for a launch's row
// count, or apply a setting to all of them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "decode.cuh"

namespace mg {
template <typename WT, int NB>
size_t decode_static_smem_nb();
template <typename WT, int NB>
cudaError_t decode_prepare_nb(size_t dynamic_smem);
template <typename WT, int NB>
int decode_occupancy_nb(size_t smem);
template <typename WT, int NB>
cudaError_t decode_launch_nb(const DecodeParams &p, int grid, size_t smem, cudaStream_t stream, bool cooperative);

static_assert(kMaxRows == 8, "decode.cu dispatches row counts 1..8");

size_t decode_smem_bytes(int S, int xs_floats, int L) {
    return 128 + static_cast<size_t>(S) * kStageBytes + static_cast<size_t>(xs_floats) * 4 + 2 * S * 8 +
           static_cast<size_t>(L) * sizeof(LayerPtrs);
}

// Largest static shared memory over the row counts.
template <typename WT>
size_t decode_static_smem() {
    return std::max({decode_static_smem_nb<WT, 1>(), decode_static_smem_nb<WT, 2>(), decode_static_smem_nb<WT, 3>(),
                     decode_static_smem_nb<WT, 4>(), decode_static_smem_nb<WT, 5>(), decode_static_smem_nb<WT, 6>(),
                     decode_static_smem_nb<WT, 7>(), decode_static_smem_nb<WT, 8>()});
}

template <typename WT>
static cudaError_t decode_prepare_all(size_t dynamic_smem) {
    cudaError_t e = cudaSuccess;
    if ((e = decode_prepare_nb<WT, 1>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 2>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 3>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 4>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 5>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 6>(dynamic_smem)) != cudaSuccess) return e;
    if ((e = decode_prepare_nb<WT, 7>(dynamic_smem)) != cudaSuccess) return e;
    return decode_prepare_nb<WT, 8>(dynamic_smem);
}

template <typename WT>
cudaError_t decode_prepare(size_t dynamic_smem) {
    // The attribute is the kernel's allowance on this device, shared by every
    // model of the process: it is only ever raised, so that a model created
    // later with a smaller stage cannot make an earlier model's launches fail.
    static std::mutex mu;
    static std::map<int, size_t> allowed;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t &cur = allowed[dev];
    if (dynamic_smem <= cur) return cudaSuccess;
    e = decode_prepare_all<WT>(dynamic_smem);
    if (e == cudaSuccess) cur = dynamic_smem;
    return e;
}

// Smallest occupancy over the row counts (every launch shape must fit).
template <typename WT>
int decode_occupancy(size_t smem) {
    return std::min({decode_occupancy_nb<WT, 1>(smem), decode_occupancy_nb<WT, 2>(smem),
                     decode_occupancy_nb<WT, 3>(smem), decode_occupancy_nb<WT, 4>(smem),
                     decode_occupancy_nb<WT, 5>(smem), decode_occupancy_nb<WT, 6>(smem),
                     decode_occupancy_nb<WT, 7>(smem), decode_occupancy_nb<WT, 8>(smem)});
}

template <typename WT>
cudaError_t decode_launch(const DecodeParams &p, int grid, size_t smem, cudaStream_t stream, bool cooperative) {
    switch (p.B) {
        case 1: return decode_launch_nb<WT, 1>(p, grid, smem, stream, cooperative);
        case 2: return decode_launch_nb<WT, 2>(p, grid, smem, stream, cooperative);
        case 3: return decode_launch_nb<WT, 3>(p, grid, smem, stream, cooperative);
        case 4: return decode_launch_nb<WT, 4>(p, grid, smem, stream, cooperative);
        case 5: return decode_launch_nb<WT, 5>(p, grid, smem, stream, cooperative);
        case 6: return decode_launch_nb<WT, 6>(p, grid, smem, stream, cooperative);
        case 7: return decode_launch_nb<WT, 7>(p, grid, smem, stream, cooperative);
        case 8: return decode_launch_nb<WT, 8>(p, grid, smem, stream, cooperative);
        default: return cudaErrorInvalidValue;
    }
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

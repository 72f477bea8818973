// decode_nb2.cu -- the decode kernel (decode_kernel.cuh) for 2 batch row(s), fp32 and bf16 weights.
#include "decode_kernel.cuh"

MG_DECODE_INSTANTIATE(2)

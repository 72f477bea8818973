// decode_nb4.cu -- the decode kernel (decode_kernel.cuh) for 4 batch row(s), fp32 and bf16 weights.
#include "decode_kernel.cuh"

MG_DECODE_INSTANTIATE(4)

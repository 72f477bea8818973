// decode_nb3.cu -- the decode kernel (decode_kernel.cuh) for 3 batch row(s), fp32 and bf16 weights.
#include "decode_kernel.cuh"

MG_DECODE_INSTANTIATE(3)

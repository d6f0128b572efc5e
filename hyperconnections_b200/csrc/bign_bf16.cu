// bf16 stream instantiations of the n > 8 stream_mix_add kernels.
#define HC_T __nv_bfloat16
#define HC_SUFFIX bf16
#define HC_T_IS_F32 0
#include "bign_inst.cuh"

// bf16 stream instantiations of the mixing kernels.
#define HC_T __nv_bfloat16
#define HC_SUFFIX bf16
#define HC_T_IS_F32 0
#include "mix_inst.cuh"

// f16 stream instantiations of the n > 8 stream_mix_add kernels.
#define HC_T __half
#define HC_SUFFIX f16
#define HC_T_IS_F32 0
#include "bign_inst.cuh"

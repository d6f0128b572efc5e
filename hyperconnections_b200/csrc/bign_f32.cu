// f32 stream instantiations of the n > 8 stream_mix_add kernels.
#define HC_T float
#define HC_SUFFIX f32
#define HC_T_IS_F32 1
#include "bign_inst.cuh"

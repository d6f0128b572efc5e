// fp16 stream instantiations of the mixing kernels.
#define HC_T __half
#define HC_SUFFIX f16
#define HC_T_IS_F32 0
#include "mix_inst.cuh"

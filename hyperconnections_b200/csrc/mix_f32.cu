// fp32 stream instantiations of the mixing kernels.
#define HC_T float
#define HC_SUFFIX f32
#define HC_T_IS_F32 1
#include "mix_inst.cuh"

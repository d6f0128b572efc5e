// f32 stream instantiations of the read / mix-write kernels, forward.
#define HC_T float
#define HC_SUFFIX f32
#define HC_RW_BWD 0
#include "rw_inst.cuh"

// f16 stream instantiations of the read / mix-write kernels, forward.
#define HC_T __half
#define HC_SUFFIX f16
#define HC_RW_BWD 0
#include "rw_inst.cuh"

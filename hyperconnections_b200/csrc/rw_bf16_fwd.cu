// bf16 stream instantiations of the read / mix-write kernels, forward.
#define HC_T __nv_bfloat16
#define HC_SUFFIX bf16
#define HC_RW_BWD 0
#include "rw_inst.cuh"

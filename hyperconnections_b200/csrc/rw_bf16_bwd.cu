// bf16 stream instantiations of the read / mix-write kernels, backward.
#define HC_T __nv_bfloat16
#define HC_SUFFIX bf16
#define HC_RW_BWD 1
#include "rw_inst.cuh"

// capi.cu — library-wide C entry points (status text, ABI version).
#include "common.cuh"

extern "C" const char* hc_error_string(int code) {
  switch (code) {
    case HC_OK: return "ok";
    case HC_ERR_NULL_POINTER: return "a required pointer is NULL";
    case HC_ERR_BAD_SIZE: return "negative or out-of-range size";
    case HC_ERR_UNSUPPORTED_N: return "number of streams / matrix order n must be in 1..8";
    case HC_ERR_DTYPE: return "unsupported dtype or dtype combination";
    case HC_ERR_ALIGNMENT: return "a float32 pointer is not 4-byte aligned";
    case HC_ERR_SCRATCH: return "scratch buffer missing or too small";
    case HC_ERR_LAUNCH: return "CUDA kernel launch failed";
    case HC_ERR_TIMEOUT:
      return "a bounded wait inside an earlier kernel gave up, so that launch's outputs are incomplete "
             "(cleared by hc_wait_timeouts with reset)";
    default: return "unknown hcops status code";
  }
}

extern "C" int hc_abi_version(void) { return 7; }

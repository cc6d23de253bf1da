// Status strings and version of the C ABI (include/halftone_b200.h).
#include <cuda_runtime.h>

#include "../../include/halftone_b200.h"

extern "C" const char* hq_status_string(int status) {
  switch (status) {
    case HQ_OK:
      return "ok";
    case HQ_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, shape, stride or alignment)";
    case HQ_ERR_UNSUPPORTED:
      return "unsupported dtype, head_dim or group size";
    case HQ_ERR_WORKSPACE:
      return "workspace missing, too small or not 256-byte aligned";
    case HQ_ERR_DEVICE_TIMEOUT:
      return "a bounded device-side wait gave up";
    default:
      if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
      return "unknown status";
  }
}

extern "C" const char* hq_version(void) { return "0.1.0"; }

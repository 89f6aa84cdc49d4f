// Version, status strings and the per-thread error message of the C ABI (flash_lab_b200.h).
#include "flash_lab_b200.h"

extern "C" int flb_version(void) { return FLB_ABI_VERSION; }

extern "C" const char* flb_status_string(int status) {
  switch (status) {
    case FLB_OK:
      return "ok";
    case FLB_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case FLB_ERR_UNSUPPORTED:
      return "unsupported input";
    case FLB_ERR_MISALIGNED:
      return "misaligned pointer or stride";
    case FLB_ERR_CUDA:
      return "CUDA error";
    case FLB_ERR_WORKSPACE:
      return "workspace too small";
    case FLB_ERR_NO_DEVICE:
      return "no sm_100 device";
    default:
      return "unknown status";
  }
}

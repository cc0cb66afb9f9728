// C-ABI entry points: argument validation, workspace layout and kernel orchestration.
#include "gdn2_common.cuh"

extern "C" const char* gdn2_status_string(gdn2_status status) {
  switch (status) {
    case GDN2_OK: return "ok";
    case GDN2_ERR_INVALID_ARGUMENT: return "invalid argument";
    case GDN2_ERR_CUDA: return "CUDA error";
    case GDN2_ERR_UNSUPPORTED: return "unsupported configuration";
  }
  return "unknown status";
}

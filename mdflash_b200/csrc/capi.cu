// Status strings and version of the ddtree_b200 C ABI.
#include "common.cuh"

extern "C" const char* ddt_error_string(int code) {
  switch (code) {
    case DDT_OK: return "ok";
    case DDT_ERR_INVALID: return "invalid argument";
    case DDT_ERR_CAPACITY: return "exceeds a compiled limit";
    case DDT_ERR_DTYPE: return "unsupported element type";
    case DDT_ERR_ALIGN: return "misaligned pointer or stride";
    case DDT_ERR_CUDA: return "CUDA runtime or launch error";
    case DDT_ERR_TIMEOUT: return "bounded device wait expired";
    case DDT_ERR_WORKSPACE: return "workspace too small";
    case DDT_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the fixed no-alloc array holds";
    default: return "unknown error";
  }
}

extern "C" int ddt_version(void) { return 1; }

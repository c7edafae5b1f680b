// Status strings, version and error bookkeeping of the C ABI.
#include "common.cuh"

namespace sb {
namespace {
thread_local int g_last_cuda_error = 0;
}
void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
}  // namespace sb

extern "C" SB_API const char *sb_status_string(int status) {
  switch (status) {
    case SB_OK: return "ok";
    case SB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SB_ERR_UNSUPPORTED: return "unsupported shape, dtype or layout";
    case SB_ERR_CUDA: return "CUDA error (see sb_last_cuda_error)";
    case SB_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case SB_ERR_TOO_LARGE: return "problem too large for one launch";
    default: return "unknown status";
  }
}

extern "C" SB_API int sb_version(void) { return 100; }

extern "C" SB_API int sb_last_cuda_error(void) { return sb::g_last_cuda_error; }

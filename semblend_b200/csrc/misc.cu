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

// ---------------------------------------------------------------------------
// Self-test of the bounded-wait machinery every pipelined kernel relies on:
// one CTA waits on an mbarrier that nothing ever arrives on, gives up after
// `max_cycles`, records `code` in *status and returns normally.
// ---------------------------------------------------------------------------
#include "tcgen05.cuh"

namespace sb {
namespace {
__global__ void wait_timeout_selftest_kernel(int *status, long long max_cycles, int code) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  const tc::Abort ab{&abort_flag, status};
  if (threadIdx.x == 0) {
    const bool ok = tc::mbar_wait(&bar, 0, ab, code, max_cycles);
    if (ok) atomicExch(status, -1);  // cannot happen: nothing arrives
  }
  __syncthreads();
}
}  // namespace
}  // namespace sb

extern "C" SB_API int sb_selftest_wait_timeout(int32_t *status, int64_t max_cycles, void *stream) {
  if (status == nullptr || max_cycles <= 0) return SB_ERR_INVALID_ARGUMENT;
  sb::wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status, max_cycles, 7);
  return sb::launch_status();
}

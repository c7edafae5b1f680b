// Status strings, version, error bookkeeping and kernel timing of the C ABI.
#include <map>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "prof.cuh"

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

// ---------------------------------------------------------------------------
// Dominant-kernel timing
// ---------------------------------------------------------------------------
namespace sb {
namespace {
std::mutex g_prof_mu;
bool g_prof_on = false;
int g_prof_used = 0;
std::vector<cudaEvent_t> g_prof_ev;  // pairs: before, after
}  // namespace

int prof_before(cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof_on || 2 * (g_prof_used + 1) > (int)g_prof_ev.size()) return -1;
  const int slot = g_prof_used++;
  cudaEventRecord(g_prof_ev[2 * slot], st);
  return slot;
}

void prof_after(int slot, cudaStream_t st) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEventRecord(g_prof_ev[2 * slot + 1], st);
}
}  // namespace sb

extern "C" SB_API int sb_profile_start(int32_t max_launches) {
  if (max_launches <= 0 || max_launches > (1 << 20)) return SB_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(sb::g_prof_mu);
  while ((int)sb::g_prof_ev.size() < 2 * max_launches) {
    cudaEvent_t e;
    cudaError_t r = cudaEventCreate(&e);
    if (r != cudaSuccess) {
      sb::set_last_cuda_error(r);
      return SB_ERR_CUDA;
    }
    sb::g_prof_ev.push_back(e);
  }
  sb::g_prof_used = 0;
  sb::g_prof_on = true;
  return SB_OK;
}

extern "C" SB_API int sb_profile_stop(float *total_ms, int32_t *n_launches) {
  std::lock_guard<std::mutex> lk(sb::g_prof_mu);
  sb::g_prof_on = false;
  float total = 0.f;
  for (int i = 0; i < sb::g_prof_used; ++i) {
    cudaError_t r = cudaEventSynchronize(sb::g_prof_ev[2 * i + 1]);
    float ms = 0.f;
    if (r == cudaSuccess) r = cudaEventElapsedTime(&ms, sb::g_prof_ev[2 * i], sb::g_prof_ev[2 * i + 1]);
    if (r != cudaSuccess) {
      sb::set_last_cuda_error(r);
      return SB_ERR_CUDA;
    }
    total += ms;
  }
  if (total_ms) *total_ms = total;
  if (n_launches) *n_launches = sb::g_prof_used;
  sb::g_prof_used = 0;
  return SB_OK;
}

namespace sb {
int ensure_dynamic_smem(const void *func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void *, int>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({func, dev});
  if (it != done.end() && it->second >= bytes) return SB_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  done[{func, dev}] = bytes;
  return SB_OK;
}
}  // namespace sb

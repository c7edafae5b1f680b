// Optional CUDA-event timing of the dominant kernel of each C-ABI call
// (sb_profile_start / sb_profile_stop): events are recorded on the launch
// stream immediately before and after that kernel.
#pragma once

#include <cuda_runtime.h>

namespace sb {
// Record the "before" event of the next dominant launch on `st` (no-op when
// profiling is off).  Returns a slot to pass to prof_after, or -1.
int prof_before(cudaStream_t st);
void prof_after(int slot, cudaStream_t st);
}  // namespace sb

// Shared helpers for the semblend_b200 CUDA sources (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/semblend_b200.h"

namespace sb {

// Records the last CUDA error seen on this host thread (sb_last_cuda_error).
void set_last_cuda_error(cudaError_t e);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

// Programmatic dependent launch (off by default: measured neutral on one GPU
// and slower when an NCCL exchange of a pipelined search runs next to the
// search kernels, whose early-launched CTAs then hold SMs while they wait).
#ifndef SB_PDL
#define SB_PDL 0
#endif

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// (prologue, TMEM allocation, barrier set-up) while the previous kernel on its
// stream finishes; it must call pdl_wait() before touching anything that
// kernel writes or reads.  pdl_launch_dependents() lets the next such kernel
// be scheduled early.  Without a programmatic predecessor both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = SB_PDL ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device):
// returns SB_OK or SB_ERR_CUDA.  Setting it on every call costs launch latency.
int ensure_dynamic_smem(const void *func, int bytes);

inline int elem_bytes(int dtype) {
  switch (dtype) {
    case SB_DTYPE_F32: return 4;
    case SB_DTYPE_F16: return 2;
    case SB_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// ---------------------------------------------------------------------------
// Element conversions to / from fp32.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f32(float x) { return x; }
  static __device__ __forceinline__ float from_f32(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};

// Raw storage of N bytes with natural alignment (N in {2,4,8,16}).
template <int N> struct RawBytes;
template <> struct RawBytes<2> { using type = uint16_t; };
template <> struct RawBytes<4> { using type = uint32_t; };
template <> struct RawBytes<8> { using type = uint2; };
template <> struct RawBytes<16> { using type = uint4; };

// A vector of VEC elements of T, loaded / stored with one instruction.
template <typename T, int VEC> struct alignas(VEC * sizeof(T)) Vec {
  static constexpr int kBytes = VEC * (int)sizeof(T);
  using Raw = typename RawBytes<kBytes>::type;
  T e[VEC];
};

// Streaming (evict-first) loads and stores: every row is touched once.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(Vec<T, VEC> &v, const T *p) {
  using Raw = typename Vec<T, VEC>::Raw;
  *reinterpret_cast<Raw *>(&v) = __ldcs(reinterpret_cast<const Raw *>(p));
}
template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T *p, const Vec<T, VEC> &v) {
  using Raw = typename Vec<T, VEC>::Raw;
  __stcs(reinterpret_cast<Raw *>(p), *reinterpret_cast<const Raw *>(&v));
}

__device__ __forceinline__ int64_t load_index(const void *p, int64_t i, int dtype) {
  return dtype == SB_INDEX_I64 ? reinterpret_cast<const int64_t *>(p)[i]
                               : (int64_t) reinterpret_cast<const int32_t *>(p)[i];
}

}  // namespace sb

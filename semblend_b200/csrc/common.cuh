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

// Masked QKV projection: out[rows[i], :] = x[rows[i], :] @ w^T + b (sm_100a).
//
// The reference computes the full GEMM for every position and zeroes the
// reuse rows afterwards (semblend_core/triton_kernels.py:366-448, wrapper
// :451-522).  Here only the compute rows are multiplied:
//   1. gather:  the compute rows of x are copied into a compact workspace
//               (16-byte vector copies; R x hidden elements),
//   2. GEMM:    a persistent warp-specialised tcgen05 kernel, M = 128 compact
//               rows x N = 256 output features per tile, K streamed in 64-wide
//               stages by TMA (128-byte swizzle) for both operands, fp32
//               accumulators double-buffered in TMEM,
//   3. epilogue: bias added in fp32, the row scattered back to its original
//               position in the caller's (zero-initialised) output.
// fp32 inputs, and 16-bit inputs whose rows are not 16-byte aligned (hidden
// sizes not a multiple of 8), run on a CUDA-core tiled kernel instead.
#include <algorithm>

#include "common.cuh"
#include "prof.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace sb {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kAStage = kBM * 128;  // 16 KB
constexpr int kBStage = kBN * 128;  // 32 KB
constexpr int kThreads = 192;       // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kSmem = 1024 + kStages * (kAStage + kBStage) + 256;
constexpr long long kWaitCycles = 2000000000LL;

struct GemmParams {
  int R, N, K;
  int m_tiles, n_tiles, k_blocks;
  const int32_t *rows;  // compact row -> output row
  const void *bias;     // [N] or null, element type T
  void *out;            // [*, ldo] element type T
  int64_t ldo;
  uint32_t idesc;
  int *status;
};

template <typename T>
__global__ void gather_rows_kernel(const T *__restrict__ x, int64_t ldx, const int32_t *__restrict__ rows, int R,
                                   int K, T *__restrict__ xc) {
  // one warp per compact row, 16-byte vectors (K * sizeof(T) is a multiple of 16)
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= R) return;
  const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)rows[w] * ldx);
  uint4 *dst = reinterpret_cast<uint4 *>(xc + w * (int64_t)K);
  const int nv = K * (int)sizeof(T) / 16;
  for (int i = lane; i < nv; i += 32) dst[i] = src[i];
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_rows_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;
  uint8_t *sB = sA + kStages * kAStage;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + kStages * kBStage);
  uint64_t *full = bars, *empty = bars + kStages;
  uint64_t *acc_full = bars + 2 * kStages, *acc_empty = acc_full + 2, *final_bar = acc_full + 4;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_full + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(acc_full + 6);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) tc::mbar_init(&full[s], 1), tc::mbar_init(&empty[s], 1);
    tc::mbar_init(&acc_full[0], 1), tc::mbar_init(&acc_full[1], 1);
    tc::mbar_init(&acc_empty[0], 4), tc::mbar_init(&acc_empty[1], 4);
    tc::mbar_init(final_bar, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_holder, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const tc::Abort ab{abort_flag, P.status};
  volatile int never = 0;
  const tc::Abort drain{&never, nullptr};
  const int64_t n_units = (int64_t)P.m_tiles * P.n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int mt = (int)(u % P.m_tiles), nt = (int)(u / P.m_tiles);
        for (int kb = 0; kb < P.k_blocks; ++kb) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1;
          if (!tc::mbar_wait(&empty[s], ph ^ 1, ab, 2, kWaitCycles)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&full[s], kAStage + kBStage);
          tc::tma_load_2d(sA + s * kAStage, &tmA, &full[s], kb * kBK, mt * kBM);
          tc::tma_load_2d(sB + s * kBStage, &tmB, &full[s], kb * kBK, nt * kBN);
          ++it;
        }
      }
      const uint32_t n_out = it < (uint32_t)kStages ? it : (uint32_t)kStages;
      for (uint32_t i = it - n_out; i < it; ++i)
        tc::mbar_wait(&full[i % kStages], (i / kStages) & 1, drain, 0, kWaitCycles);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, ai = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const uint32_t b = ai & 1;
        if (!tc::mbar_wait(&acc_empty[b], ((ai >> 1) & 1) ^ 1, ab, 3, kWaitCycles)) break;
        tc::fence_after_sync();
        for (int kb = 0; kb < P.k_blocks; ++kb) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1;
          if (!tc::mbar_wait(&full[s], ph, ab, 3, kWaitCycles)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::mma_bf16_ss(tmem + b * kBN, tc::desc_kmajor_sw128(sA + s * kAStage, kk * 32),
                            tc::desc_kmajor_sw128(sB + s * kBStage, kk * 32), P.idesc, (kb | kk) != 0);
          tc::mma_commit(&empty[s]);
          ++it;
        }
        if (!ok) break;
        tc::mma_commit(&acc_full[b]);
        ++ai;
      }
      tc::mma_commit(final_bar);
      tc::mbar_wait(final_bar, 0, drain, 0, kWaitCycles);
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    uint32_t ai = 0;
    for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
      const int mt = (int)(u % P.m_tiles), nt = (int)(u / P.m_tiles);
      const uint32_t b = ai & 1;
      if (!tc::mbar_wait(&acc_full[b], (ai >> 1) & 1, ab, 4, kWaitCycles)) break;
      tc::fence_after_sync();
      const int m = mt * kBM + row;
      const bool active = m < P.R;
      T *dst = active ? reinterpret_cast<T *>(P.out) + (int64_t)P.rows[m] * P.ldo : nullptr;
      const T *bias = reinterpret_cast<const T *>(P.bias);
      const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + b * kBN;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t r[32];
        tc::tmem_ld32(base + c, r);
        tc::tmem_ld_wait();
        const int n0 = nt * kBN + c;
        if (active && n0 < P.N) {
          if (n0 + 32 <= P.N) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float v0 = __uint_as_float(r[2 * i]), v1 = __uint_as_float(r[2 * i + 1]);
              if (bias) v0 += Elem<T>::to_f32(bias[n0 + 2 * i]), v1 += Elem<T>::to_f32(bias[n0 + 2 * i + 1]);
              T t0 = Elem<T>::from_f32(v0), t1 = Elem<T>::from_f32(v1);
              pk[i] = (uint32_t)(*reinterpret_cast<uint16_t *>(&t0)) |
                      ((uint32_t)(*reinterpret_cast<uint16_t *>(&t1)) << 16);
            }
            uint4 *d4 = reinterpret_cast<uint4 *>(dst + n0);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (n0 + i < P.N) {
                float v = __uint_as_float(r[i]);
                if (bias) v += Elem<T>::to_f32(bias[n0 + i]);
                dst[n0 + i] = Elem<T>::from_f32(v);
              }
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
      ++ai;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// CUDA-core path (fp32, and 16-bit shapes the TMA path cannot take): 64 x 64
// output tiles, 256 threads each computing 4 x 4 outputs, fp32 accumulation,
// one rounding to T after the bias.
template <typename T>
__global__ void __launch_bounds__(256) gemm_rows_simt_kernel(const T *__restrict__ x, int64_t ldx,
                                                             const T *__restrict__ w, int64_t ldw,
                                                             const T *__restrict__ bias,
                                                             const int32_t *__restrict__ rows, int R, int N, int K,
                                                             T *__restrict__ out, int64_t ldo) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i % 16, mm = i / 16;
      const int m = m0 + mm, n = n0 + mm, k = k0 + kk;
      As[kk][mm] = (m < R && k < K) ? Elem<T>::to_f32(x[(int64_t)rows[m] * ldx + k]) : 0.f;
      Bs[kk][mm] = (n < N && k < K) ? Elem<T>::to_f32(w[(int64_t)n * ldw + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(As[kk][ty * 4 + i], Bs[kk][tx * 4 + j], acc[i][j]);
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= R) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N)
        out[(int64_t)rows[m] * ldo + n] = Elem<T>::from_f32(acc[i][j] + (bias ? Elem<T>::to_f32(bias[n]) : 0.f));
    }
  }
}

template <typename T>
int launch_simt(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *bias, const int32_t *rows,
                int R, int N, int K, void *out, int64_t ldo, cudaStream_t st) {
  dim3 grid((unsigned)((R + 63) / 64), (unsigned)((N + 63) / 64));
  const int slot = prof_before(st);
  gemm_rows_simt_kernel<T><<<grid, 256, 0, st>>>(reinterpret_cast<const T *>(x), ldx, reinterpret_cast<const T *>(w),
                                                 ldw, reinterpret_cast<const T *>(bias), rows, R, N, K,
                                                 reinterpret_cast<T *>(out), ldo);
  prof_after(slot, st);
  return launch_status();
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

template <typename T>
int launch_tc(const T *x, int64_t ldx, const T *w, int64_t ldw, const T *bias, const int32_t *rows, int R, int N,
              int K, T *out, int64_t ldo, T *xc, int *status, CUtensorMapDataType dt, uint32_t fmt,
              cudaStream_t st) {
  gather_rows_kernel<T><<<(unsigned)(((int64_t)R * 32 + 255) / 256), 256, 0, st>>>(x, ldx, rows, R, K, xc);
  int s = launch_status();
  if (s != SB_OK) return s;
  CUtensorMap ta, tb;
  if (!make_tmap_16_2d(&ta, dt, xc, K, R, (uint64_t)K * sizeof(T), kBK, kBM) ||
      !make_tmap_16_2d(&tb, dt, w, K, N, (uint64_t)ldw * sizeof(T), kBK, kBN))
    return SB_ERR_CUDA;
  GemmParams P;
  P.R = R, P.N = N, P.K = K;
  P.m_tiles = (R + kBM - 1) / kBM;
  P.n_tiles = (N + kBN - 1) / kBN;
  P.k_blocks = (K + kBK - 1) / kBK;
  P.rows = rows, P.bias = bias, P.out = out, P.ldo = ldo;
  P.idesc = tc::idesc_f16(kBM, kBN, fmt, 0);
  P.status = status;
  if (ensure_dynamic_smem(reinterpret_cast<const void *>(gemm_rows_kernel<T>), kSmem) != SB_OK) return SB_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(sm_count(), (int64_t)P.m_tiles * P.n_tiles);
  const int slot = prof_before(st);
  gemm_rows_kernel<T><<<grid, kThreads, kSmem, st>>>(ta, tb, P);
  prof_after(slot, st);
  return launch_status();
}

}  // namespace
}  // namespace sb

extern "C" SB_API int64_t sb_masked_linear_workspace_bytes(int32_t n_rows, int32_t in_features, int32_t dtype) {
  const int es = sb::elem_bytes(dtype);
  if (es == 0 || n_rows < 0 || in_features <= 0) return -1;
  return dtype == SB_DTYPE_F32 ? 0 : (int64_t)n_rows * in_features * es;
}

extern "C" SB_API int sb_masked_linear(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *bias,
                                       const int32_t *rows, int32_t n_rows, int32_t out_features,
                                       int32_t in_features, void *out, int64_t ldo, int32_t dtype, void *workspace,
                                       int64_t workspace_bytes, int32_t *status, void *stream) {
  using namespace sb;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (n_rows < 0 || out_features <= 0 || in_features <= 0) return SB_ERR_INVALID_ARGUMENT;
  if (n_rows == 0) return SB_OK;
  if (!x || !w || !rows || !out || !status) return SB_ERR_INVALID_ARGUMENT;
  if (ldx < in_features || ldw < in_features || ldo < out_features) return SB_ERR_INVALID_ARGUMENT;
  const int es = elem_bytes(dtype);
  if (es == 0) return SB_ERR_UNSUPPORTED;
  if (dtype == SB_DTYPE_F32)
    return launch_simt<float>(x, ldx, w, ldw, bias, rows, n_rows, out_features, in_features, out, ldo, st);
  // tensor-core path: 16-byte aligned rows and K a multiple of 8 elements
  if ((in_features * es) % 16 || (ldx * es) % 16 || (ldw * es) % 16 || (ldo * es) % 16 ||
      (reinterpret_cast<uintptr_t>(x) % 16) || (reinterpret_cast<uintptr_t>(w) % 16) ||
      (reinterpret_cast<uintptr_t>(out) % 16)) {
    if (dtype == SB_DTYPE_BF16)
      return launch_simt<__nv_bfloat16>(x, ldx, w, ldw, bias, rows, n_rows, out_features, in_features, out, ldo, st);
    return launch_simt<__half>(x, ldx, w, ldw, bias, rows, n_rows, out_features, in_features, out, ldo, st);
  }
  const int64_t need = (int64_t)n_rows * in_features * es;
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) % 16))
    return SB_ERR_WORKSPACE_TOO_SMALL;
  if (dtype == SB_DTYPE_BF16)
    return launch_tc<__nv_bfloat16>(
        reinterpret_cast<const __nv_bfloat16 *>(x), ldx, reinterpret_cast<const __nv_bfloat16 *>(w), ldw,
        reinterpret_cast<const __nv_bfloat16 *>(bias), rows, n_rows, out_features, in_features,
        reinterpret_cast<__nv_bfloat16 *>(out), ldo, reinterpret_cast<__nv_bfloat16 *>(workspace), status,
        CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 1u, st);
  return launch_tc<__half>(reinterpret_cast<const __half *>(x), ldx, reinterpret_cast<const __half *>(w), ldw,
                           reinterpret_cast<const __half *>(bias), rows, n_rows, out_features, in_features,
                           reinterpret_cast<__half *>(out), ldo, reinterpret_cast<__half *>(workspace), status,
                           CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 0u, st);
}

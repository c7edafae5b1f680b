// Chunk-hash alignment on the GPU (sm_100a).
//
// The reference aligns a target token sequence to a donor one on the host
// (semblend_core/alignment.py:120-268): every full chunk of `chunk` tokens is
// hashed with SHA-256 over its ids packed as little-endian uint32 (first 128
// bits kept), each target chunk in order takes the first unused donor chunk
// with the same hash, and an optional context gate drops matches with no
// matched neighbour; the result is expanded into per-position pairs.  Here:
//   1. chunk_sha256_kernel   one thread per full chunk: SHA-256 (FIPS 180-4)
//                            of the chunk's 4 * chunk bytes;
//   2. chunk_match_kernel    one thread per target chunk: its rank among the
//                            earlier target chunks with the same digest picks
//                            the donor chunk of the same rank among donor
//                            chunks with that digest (= the greedy first-unused
//                            rule of the reference, computed in parallel), then
//                            the context gate on its neighbours' matches;
//   3. chunk_pairs_kernel    one CTA: a block-wide scan over the matched chunks
//                            and the (donor, target) position pairs written
//                            straight into the inject kernel's input arrays,
//                            with their count.
// The SHA-256 round constants and initial hash are computed on the host from
// their definition (fractional parts of the cube / square roots of the first
// 64 / 8 primes) and copied to constant memory once per device.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace sb {
namespace {

__constant__ uint32_t c_sha_k[64];
__constant__ uint32_t c_sha_h0[8];

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

__device__ __forceinline__ void sha256_block(uint32_t (&h)[8], const uint32_t (&m)[16]) {
  uint32_t w[64];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = m[i];
#pragma unroll
  for (int i = 16; i < 64; ++i) {
    const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + c_sha_k[i] + w[i];
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + maj;
    hh = g, g = f, f = e, e = d + t1, d = c, c = b, b = a, a = t1 + t2;
  }
  h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
}

// Digest (first 128 bits, as four big-endian words) of every full chunk.
template <typename I>
__global__ void chunk_sha256_kernel(const I *__restrict__ tokens, int chunk, int64_t n_chunks,
                                    uint32_t *__restrict__ digests) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  const I *t = tokens + c * chunk;
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = c_sha_h0[i];
  uint32_t m[16];
  // message: 4 bytes per token (little-endian uint32), SHA-256 reads big-endian words
  for (int base = 0; base < chunk; base += 16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = base + i < chunk ? bswap((uint32_t)t[base + i]) : 0u;
    const int n = chunk - base;
    if (n >= 16) {
      sha256_block(h, m);
    } else {  // tail block (chunk not a multiple of 16 tokens): padding follows the data
      m[n] = 0x80000000u;
      if (n <= 13) {
        m[14] = (uint32_t)(((uint64_t)chunk * 32) >> 32);
        m[15] = (uint32_t)((uint64_t)chunk * 32);
        sha256_block(h, m);
      } else {
        sha256_block(h, m);
#pragma unroll
        for (int i = 0; i < 16; ++i) m[i] = 0;
        m[14] = (uint32_t)(((uint64_t)chunk * 32) >> 32);
        m[15] = (uint32_t)((uint64_t)chunk * 32);
        sha256_block(h, m);
      }
      break;
    }
  }
  if (chunk % 16 == 0) {  // data filled whole blocks: one padding block
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = 0;
    m[0] = 0x80000000u;
    m[14] = (uint32_t)(((uint64_t)chunk * 32) >> 32);
    m[15] = (uint32_t)((uint64_t)chunk * 32);
    sha256_block(h, m);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) digests[c * 4 + i] = h[i];
}

__device__ __forceinline__ bool same(const uint32_t *a, const uint32_t *b) {
  return a[0] == b[0] && a[1] == b[1] && a[2] == b[2] && a[3] == b[3];
}

// Phase 1 (no gate): target chunk t takes the donor chunk whose rank among
// donor chunks with t's digest equals t's rank among target chunks with it.
__device__ int phase1_match(const uint32_t *__restrict__ dd, int nd, const uint32_t *__restrict__ td, int t) {
  const uint32_t *me = td + 4 * t;
  int rank = 0;
  for (int u = 0; u < t; ++u) rank += same(td + 4 * u, me);
  for (int d = 0; d < nd; ++d) {
    if (same(dd + 4 * d, me)) {
      if (rank == 0) return d;
      --rank;
    }
  }
  return -1;
}

// Final match of target chunk t; with the context gate a match survives only
// if a neighbouring target chunk matched in phase 1 (each thread recomputes
// its neighbours' phase-1 result, so no pass over the whole array is needed).
__global__ void chunk_match_kernel(const uint32_t *__restrict__ dd, int nd, const uint32_t *__restrict__ td, int nt,
                                   int gate, int32_t *__restrict__ match) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nt) return;
  int m = phase1_match(dd, nd, td, t);
  if (gate && m >= 0) {
    const bool left = t > 0 && phase1_match(dd, nd, td, t - 1) >= 0;
    const bool right = t + 1 < nt && phase1_match(dd, nd, td, t + 1) >= 0;
    if (!left && !right) m = -1;
  }
  match[t] = m;
}

// The pair arrays: matched chunk i (in target order) owns pairs
// [i * chunk, (i + 1) * chunk).  One CTA, a block-wide scan per 1024 chunks.
__global__ void chunk_pairs_kernel(const int32_t *__restrict__ match, int nt, int chunk,
                                   int32_t *__restrict__ donor_pos, int32_t *__restrict__ target_pos,
                                   int64_t *__restrict__ n_pairs) {
  __shared__ int warp_sum[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int base = 0; base < nt; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const int m = t < nt ? match[t] : -1;
    const int f = m >= 0;
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    if (lane == 0) warp_sum[wid] = __popc(bal);
    __syncthreads();
    int off = carry, tot = 0;
    for (int i = 0; i < nw; ++i) {
      if (i < wid) off += warp_sum[i];
      tot += warp_sum[i];
    }
    off += __popc(bal & ((1u << lane) - 1));
    if (f) {
      for (int i = 0; i < chunk; ++i) {
        donor_pos[(int64_t)off * chunk + i] = m * chunk + i;
        target_pos[(int64_t)off * chunk + i] = t * chunk + i;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_pairs = (int64_t)carry * chunk;
}

// SHA-256 constants from their definition, on the host with 64-bit-mantissa
// arithmetic, copied to each device once.
int upload_constants() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return SB_OK;
  uint32_t k[64], h0[8];
  int n = 0;
  for (int p = 2; n < 64; ++p) {
    bool prime = true;
    for (int q = 2; q * q <= p; ++q) prime = prime && (p % q != 0);
    if (!prime) continue;
    const long double r3 = cbrtl((long double)p), r2 = sqrtl((long double)p);
    k[n] = (uint32_t)((r3 - floorl(r3)) * 4294967296.0L);
    if (n < 8) h0[n] = (uint32_t)((r2 - floorl(r2)) * 4294967296.0L);
    ++n;
  }
  e = cudaMemcpyToSymbol(c_sha_k, k, sizeof(k));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_sha_h0, h0, sizeof(h0));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  done[dev] = true;
  return SB_OK;
}

}  // namespace
}  // namespace sb

extern "C" SB_API int sb_chunk_digests(const void *tokens, int32_t token_dtype, int64_t n_tokens, int32_t chunk,
                                       uint32_t *digests, void *stream) {
  using namespace sb;
  if (n_tokens < 0 || chunk <= 0) return SB_ERR_INVALID_ARGUMENT;
  if (token_dtype != SB_INDEX_I32 && token_dtype != SB_INDEX_I64) return SB_ERR_UNSUPPORTED;
  const int64_t n_chunks = n_tokens / chunk;
  if (n_chunks == 0) return SB_OK;
  if (!tokens || !digests) return SB_ERR_INVALID_ARGUMENT;
  const int s = upload_constants();
  if (s != SB_OK) return s;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((n_chunks + 127) / 128);
  if (token_dtype == SB_INDEX_I32)
    chunk_sha256_kernel<int32_t><<<grid, 128, 0, st>>>(static_cast<const int32_t *>(tokens), chunk, n_chunks,
                                                       digests);
  else
    chunk_sha256_kernel<int64_t><<<grid, 128, 0, st>>>(static_cast<const int64_t *>(tokens), chunk, n_chunks,
                                                       digests);
  return launch_status();
}

extern "C" SB_API int sb_chunk_align(const uint32_t *donor_digests, int32_t n_donor_chunks,
                                     const uint32_t *target_digests, int32_t n_target_chunks, int32_t chunk,
                                     int32_t context_gate, int32_t *match, int32_t *donor_positions,
                                     int32_t *target_positions, int64_t *n_pairs, void *stream) {
  using namespace sb;
  if (n_donor_chunks < 0 || n_target_chunks < 0 || chunk <= 0) return SB_ERR_INVALID_ARGUMENT;
  if ((int64_t)n_target_chunks * chunk > 0x7fffffffLL || (int64_t)n_donor_chunks * chunk > 0x7fffffffLL)
    return SB_ERR_TOO_LARGE;
  if (!n_pairs || (n_target_chunks > 0 && (!target_digests || !match || !donor_positions || !target_positions)))
    return SB_ERR_INVALID_ARGUMENT;
  if (n_donor_chunks > 0 && !donor_digests) return SB_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (n_target_chunks == 0) {
    cudaError_t e = cudaMemsetAsync(n_pairs, 0, sizeof(int64_t), st);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return SB_ERR_CUDA;
    }
    return SB_OK;
  }
  chunk_match_kernel<<<(unsigned)((n_target_chunks + 127) / 128), 128, 0, st>>>(
      donor_digests, n_donor_chunks, target_digests, n_target_chunks, context_gate ? 1 : 0, match);
  int s = launch_status();
  if (s != SB_OK) return s;
  chunk_pairs_kernel<<<1, 1024, 0, st>>>(match, n_target_chunks, chunk, donor_positions, target_positions,
                                         n_pairs);
  return launch_status();
}

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
//   2. chunk_match_kernel    one CTA per request, one thread per target chunk:
//                            its rank among the earlier target chunks with the
//                            same digest picks the donor chunk of the same
//                            rank among donor chunks with that digest (= the
//                            greedy first-unused rule of the reference,
//                            computed in parallel), then the context gate on
//                            its neighbours' matches;
//   3. chunk_pairs_kernel    a few target chunks per CTA: the matched chunks'
//                            (donor, target) position pairs written straight
//                            into the inject kernel's input arrays (-1 after
//                            the last), with their count.
// The SHA-256 round constants and initial hash are computed on the host from
// their definition (fractional parts of the cube / square roots of the first
// 64 / 8 primes) and copied to constant memory once per device.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "prof.cuh"

namespace sb {
namespace {

// chunks are few (one per 256 tokens): small CTAs spread them over the SMs
constexpr int kShaThreads = 32;

__constant__ uint32_t c_sha_k[64];
__constant__ uint32_t c_sha_h0[8];

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
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
// One loop over the message blocks (data, then the 0x80 byte and the bit
// length as FIPS 180-4 pads them), so the compression is inlined once; the
// ids of the next block are loaded while the current one is compressed.
template <typename I>
__global__ void __launch_bounds__(kShaThreads) chunk_sha256_kernel(const I *__restrict__ tokens, int chunk,
                                                                   int64_t n_chunks, uint32_t *__restrict__ digests) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  const I *t = tokens + c * chunk;
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = c_sha_h0[i];
  // message: 4 bytes per token (little-endian uint32) then the padding; SHA-256 reads big-endian words
  const int n_blocks = (chunk + 2) / 16 + 1;  // 4 * chunk + 9 bytes, rounded up to 64-byte blocks
  const uint64_t bits = (uint64_t)chunk * 32;
  uint32_t m[16], nxt[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) nxt[i] = i < chunk ? (uint32_t)t[i] : 0u;
  for (int blk = 0; blk < n_blocks; ++blk) {
    const int base = blk * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int g = base + i;
      m[i] = g < chunk ? bswap(nxt[i]) : (g == chunk ? 0x80000000u : 0u);
    }
    if (blk == n_blocks - 1) {
      m[14] = (uint32_t)(bits >> 32);
      m[15] = (uint32_t)bits;
    }
    if (base + 16 < chunk) {
#pragma unroll
      for (int i = 0; i < 16; ++i) nxt[i] = base + 16 + i < chunk ? (uint32_t)t[base + 16 + i] : 0u;
    }
    sha256_block(h, m);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) digests[c * 4 + i] = h[i];
}

// The requests of one launch.  Request r owns donor digests [d0, d0 + nd),
// full target chunks [t0, t0 + nt) (digests, and pair slots [t0 * chunk,
// (t0 + nt) * chunk)) and match entries [m0, m0 + nm) (its full target
// chunks, then -1 for a trailing partial chunk).  offs holds the three prefix
// arrays [3][n + 1]; NULL means one request with the counts nd1 / nt1 / nm1.
struct AlignBatch {
  const uint32_t *dd, *td;
  const int32_t *offs;
  int n, nd1, nt1, nm1, max_nt;
  int chunk, gate;
  int32_t *match, *dpos, *tpos;
  int64_t *n_pairs;
};

struct ReqRange {
  int d0, nd, t0, nt, m0, nm;
};

__device__ __forceinline__ bool req_range(const AlignBatch &B, int r, ReqRange &q) {
  if (B.offs == nullptr) {
    q = ReqRange{0, B.nd1, 0, B.nt1, 0, B.nm1};
  } else {
    const int s = B.n + 1;
    q.d0 = B.offs[r], q.nd = B.offs[r + 1] - q.d0;
    q.t0 = B.offs[s + r], q.nt = B.offs[s + r + 1] - q.t0;
    q.m0 = B.offs[2 * s + r], q.nm = B.offs[2 * s + r + 1] - q.m0;
  }
  // offsets that do not describe a request this launch was sized for: skip it
  return q.nd >= 0 && q.nt >= 0 && q.nt <= B.max_nt && q.nm >= q.nt && q.d0 >= 0 && q.t0 >= 0 && q.m0 >= 0;
}

__device__ __forceinline__ bool same(const uint32_t *a, const uint4 b) {
  return a[0] == b.x && a[1] == b.y && a[2] == b.z && a[3] == b.w;
}

constexpr int kMatchThreads = 512;
constexpr int kMatchSmemWords = 8192;  // first digest words of a request staged in shared memory (32 KB)
constexpr int kMaxTargetChunks = 65536;  // per request: the matched-chunk flags live in shared memory (8 KB)

// One CTA per request.  Phase 1 (no gate): target chunk t takes the donor
// chunk whose rank among the donor chunks with t's digest equals t's rank
// among the earlier target chunks with it (= the greedy first-unused rule).
// The scans compare the digests' first words (staged in shared memory and
// read by a warp in step, so each read is a broadcast) and the full digests
// only on a first-word hit.  Then the context gate: a match survives only if
// target chunk t - 1 or t + 1 also matched in phase 1.
__global__ void __launch_bounds__(kMatchThreads) chunk_match_kernel(const AlignBatch B) {
  __shared__ uint32_t w0[kMatchSmemWords];
  __shared__ uint32_t hit[kMaxTargetChunks / 32];
  ReqRange q;
  if (!req_range(B, blockIdx.x, q)) return;
  const uint32_t *dd = B.dd + 4LL * q.d0, *td = B.td + 4LL * q.t0;
  int32_t *match = B.match + q.m0;
  const bool staged = q.nd + q.nt <= kMatchSmemWords;
  if (staged) {
    for (int i = threadIdx.x; i < q.nd; i += kMatchThreads) w0[i] = dd[4 * i];
    for (int i = threadIdx.x; i < q.nt; i += kMatchThreads) w0[q.nd + i] = td[4 * i];
  }
  for (int i = threadIdx.x; i < (q.nt + 31) / 32; i += kMatchThreads) hit[i] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < q.nt; t += kMatchThreads) {
    const uint4 me = make_uint4(td[4 * t], td[4 * t + 1], td[4 * t + 2], td[4 * t + 3]);
    int rank = 0;
    for (int u = 0; u < t; ++u) {
      const uint32_t w = staged ? w0[q.nd + u] : td[4 * u];
      rank += w == me.x && same(td + 4 * u, me);
    }
    int m = -1;
    for (int d = 0; d < q.nd; ++d) {
      const uint32_t w = staged ? w0[d] : dd[4 * d];
      if (w == me.x && same(dd + 4 * d, me)) {
        if (rank == 0) {
          m = d;
          break;
        }
        --rank;
      }
    }
    match[t] = m;
    if (m >= 0) atomicOr(&hit[t >> 5], 1u << (t & 31));
  }
  __syncthreads();
  auto flag = [&](int t) { return (hit[t >> 5] >> (t & 31)) & 1u; };
  for (int t = threadIdx.x; t < q.nm; t += kMatchThreads) {
    if (t >= q.nt) {
      match[t] = -1;
    } else if (B.gate && flag(t) && !(t > 0 && flag(t - 1)) && !(t + 1 < q.nt && flag(t + 1))) {
      match[t] = -1;
    }
  }
}

// The pair arrays: matched chunk i of a request (in target order) owns pairs
// [i * chunk, (i + 1) * chunk) of the request's slots; the slots after its
// last matched chunk are filled with -1, unmatched chunk c taking slot
// (matched total + unmatched chunks before c).  CTA (x, r) handles
// kPairChunks consecutive target chunks of request r: it counts the matched
// chunks before its range and in total (one entry per chunk: small), then
// writes its chunks' pairs with the whole block, so the stores are coalesced.
constexpr int kPairChunks = 4;
constexpr int kPairThreads = 256;

__global__ void __launch_bounds__(kPairThreads) chunk_pairs_kernel(const AlignBatch B) {
  __shared__ int red[2][kPairThreads / 32];
  ReqRange q;
  const bool ok = req_range(B, blockIdx.y, q);
  if (!ok) {
    if (blockIdx.x == 0 && threadIdx.x == 0) B.n_pairs[blockIdx.y] = -1;
    return;
  }
  const int c0 = blockIdx.x * kPairChunks;
  if (blockIdx.x > 0 && c0 >= q.nt) return;
  const int32_t *match = B.match + q.m0;
  const int c1 = min(q.nt, c0 + kPairChunks);
  int before = 0, total = 0;
  for (int i = threadIdx.x; i < q.nt; i += kPairThreads) {
    const int f = match[i] >= 0;
    total += f;
    before += f & (i < c0);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    before += __shfl_xor_sync(0xffffffffu, before, o);
    total += __shfl_xor_sync(0xffffffffu, total, o);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[0][wid] = before, red[1][wid] = total;
  __syncthreads();
  before = 0, total = 0;
#pragma unroll
  for (int i = 0; i < kPairThreads / 32; ++i) before += red[0][i], total += red[1][i];
  const int chunk = B.chunk;
  if (blockIdx.x == 0 && threadIdx.x == 0) B.n_pairs[blockIdx.y] = (int64_t)total * chunk;
  int32_t *dpos = B.dpos + (int64_t)q.t0 * chunk, *tpos = B.tpos + (int64_t)q.t0 * chunk;
  int matched = before;
  for (int c = c0; c < c1; ++c) {
    const int m = match[c];
    const bool got = m >= 0;
    const int64_t slot = got ? matched : (int64_t)total + (c - matched);
    int32_t *dp = dpos + slot * chunk, *tp = tpos + slot * chunk;
    for (int i = threadIdx.x; i < chunk; i += kPairThreads) {
      dp[i] = got ? m * chunk + i : -1;
      tp[i] = got ? c * chunk + i : -1;
    }
    matched += got;
  }
}

// Multiset overlap of two token sequences, sum over ids of min(count in
// donor, count in target): an open-addressing table (linear probing, at most
// half full) of 64-bit ids with a donor and a target count per slot.  The
// all-ones id (-1), which marks empty slots, is counted in a slot of its own.
constexpr uint64_t kEmptyKey = ~0ull;

struct OverlapTable {
  unsigned long long *keys;  // [cap]
  unsigned *cnt;             // [cap + 1][2]: donor, target (slot cap: id -1)
  uint64_t mask;             // cap - 1 (cap a power of two)
};

__device__ __forceinline__ uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

template <typename ID, typename IT>
__global__ void overlap_count_kernel(const ID *__restrict__ donor, int64_t n_d, const IT *__restrict__ target,
                                     int64_t n_t, OverlapTable T) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_d + n_t) return;
  const bool is_t = i >= n_d;
  const uint64_t key = is_t ? (uint64_t)(int64_t)target[i - n_d] : (uint64_t)(int64_t)donor[i];
  uint64_t slot;
  if (key == kEmptyKey) {
    slot = T.mask + 1;
  } else {
    slot = mix64(key) & T.mask;
    // at most half full: the probe ends at the key or at an empty slot
    for (uint64_t n = 0; n <= T.mask; ++n) {
      const unsigned long long prev = atomicCAS(&T.keys[slot], kEmptyKey, (unsigned long long)key);
      if (prev == kEmptyKey || prev == key) break;
      slot = (slot + 1) & T.mask;
    }
  }
  atomicAdd(&T.cnt[2 * slot + (is_t ? 1 : 0)], 1u);
}

__global__ void overlap_sum_kernel(OverlapTable T, unsigned long long *__restrict__ out) {
  unsigned long long acc = 0;
  for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s <= T.mask + 1;
       s += (uint64_t)gridDim.x * blockDim.x)
    acc += min(T.cnt[2 * s], T.cnt[2 * s + 1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out, acc);
}

uint64_t overlap_capacity(int64_t n_d, int64_t n_t) {
  uint64_t cap = 1024;
  while (cap < 2 * (uint64_t)(n_d + n_t)) cap <<= 1;
  return cap;
}

int64_t overlap_workspace_bytes(int64_t n_d, int64_t n_t) {
  const uint64_t cap = overlap_capacity(n_d, n_t);
  return (int64_t)(cap * 8 + (cap + 1) * 8);
}

template <typename ID, typename IT>
void launch_overlap_count(const void *d, int64_t n_d, const void *t, int64_t n_t, const OverlapTable &T,
                          cudaStream_t st) {
  const unsigned grid = (unsigned)((n_d + n_t + 255) / 256);
  overlap_count_kernel<ID, IT><<<grid, 256, 0, st>>>(static_cast<const ID *>(d), n_d, static_cast<const IT *>(t),
                                                      n_t, T);
}

int launch_align(const AlignBatch &B, cudaStream_t st) {
  chunk_match_kernel<<<(unsigned)B.n, kMatchThreads, 0, st>>>(B);
  int s = launch_status();
  if (s != SB_OK) return s;
  const unsigned gx = (unsigned)std::max(1, (B.max_nt + kPairChunks - 1) / kPairChunks);
  chunk_pairs_kernel<<<dim3(gx, (unsigned)B.n), kPairThreads, 0, st>>>(B);
  return launch_status();
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
  const unsigned grid = (unsigned)((n_chunks + kShaThreads - 1) / kShaThreads);
  const int slot = prof_before(st);
  if (token_dtype == SB_INDEX_I32)
    chunk_sha256_kernel<int32_t><<<grid, kShaThreads, 0, st>>>(static_cast<const int32_t *>(tokens), chunk,
                                                               n_chunks, digests);
  else
    chunk_sha256_kernel<int64_t><<<grid, kShaThreads, 0, st>>>(static_cast<const int64_t *>(tokens), chunk,
                                                               n_chunks, digests);
  prof_after(slot, st);
  return launch_status();
}

extern "C" SB_API int sb_chunk_align(const uint32_t *donor_digests, int32_t n_donor_chunks,
                                     const uint32_t *target_digests, int32_t n_target_chunks, int32_t chunk,
                                     int32_t context_gate, int32_t *match, int32_t *donor_positions,
                                     int32_t *target_positions, int64_t *n_pairs, void *stream) {
  using namespace sb;
  if (n_donor_chunks < 0 || n_target_chunks < 0 || chunk <= 0) return SB_ERR_INVALID_ARGUMENT;
  if ((int64_t)n_target_chunks * chunk > 0x7fffffffLL || (int64_t)n_donor_chunks * chunk > 0x7fffffffLL ||
      n_target_chunks > kMaxTargetChunks)
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
  AlignBatch B{};
  B.dd = donor_digests, B.td = target_digests, B.offs = nullptr;
  B.n = 1, B.nd1 = n_donor_chunks, B.nt1 = n_target_chunks, B.nm1 = n_target_chunks, B.max_nt = n_target_chunks;
  B.chunk = chunk, B.gate = context_gate ? 1 : 0;
  B.match = match, B.dpos = donor_positions, B.tpos = target_positions, B.n_pairs = n_pairs;
  return launch_align(B, st);
}

extern "C" SB_API int sb_chunk_align_batch(const uint32_t *donor_digests, const uint32_t *target_digests,
                                           const int32_t *offsets, int32_t n_requests, int32_t max_target_chunks,
                                           int32_t chunk, int32_t context_gate, int32_t *match,
                                           int32_t *donor_positions, int32_t *target_positions, int64_t *n_pairs,
                                           void *stream) {
  using namespace sb;
  if (n_requests < 0 || max_target_chunks < 0 || chunk <= 0) return SB_ERR_INVALID_ARGUMENT;
  if (n_requests > 65535 || max_target_chunks > kMaxTargetChunks ||
      (int64_t)max_target_chunks * chunk > 0x7fffffffLL)
    return SB_ERR_TOO_LARGE;
  if (n_requests == 0) return SB_OK;
  if (!offsets || !match || !n_pairs || (max_target_chunks > 0 && (!target_digests || !donor_positions ||
                                                                   !target_positions)))
    return SB_ERR_INVALID_ARGUMENT;
  AlignBatch B{};
  B.dd = donor_digests, B.td = target_digests, B.offs = offsets;
  B.n = n_requests, B.max_nt = max_target_chunks;
  B.chunk = chunk, B.gate = context_gate ? 1 : 0;
  B.match = match, B.dpos = donor_positions, B.tpos = target_positions, B.n_pairs = n_pairs;
  return launch_align(B, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" SB_API int64_t sb_token_overlap_workspace_bytes(int64_t n_donor_tokens, int64_t n_target_tokens) {
  if (n_donor_tokens < 0 || n_target_tokens < 0) return SB_ERR_INVALID_ARGUMENT;
  return sb::overlap_workspace_bytes(n_donor_tokens, n_target_tokens);
}

extern "C" SB_API int sb_token_overlap(const void *donor_tokens, int32_t donor_dtype, int64_t n_donor_tokens,
                                       const void *target_tokens, int32_t target_dtype, int64_t n_target_tokens,
                                       void *workspace, int64_t workspace_bytes, int64_t *overlap, void *stream) {
  using namespace sb;
  if (n_donor_tokens < 0 || n_target_tokens < 0 || !overlap) return SB_ERR_INVALID_ARGUMENT;
  if ((donor_dtype != SB_INDEX_I32 && donor_dtype != SB_INDEX_I64) ||
      (target_dtype != SB_INDEX_I32 && target_dtype != SB_INDEX_I64))
    return SB_ERR_UNSUPPORTED;
  if (n_donor_tokens + n_target_tokens > 0x7fffffffLL) return SB_ERR_TOO_LARGE;  // 32-bit counts per id
  if ((n_donor_tokens > 0 && !donor_tokens) || (n_target_tokens > 0 && !target_tokens))
    return SB_ERR_INVALID_ARGUMENT;
  const int64_t need = overlap_workspace_bytes(n_donor_tokens, n_target_tokens);
  if (!workspace || workspace_bytes < need) return SB_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(workspace) % 8) return SB_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint64_t cap = overlap_capacity(n_donor_tokens, n_target_tokens);
  OverlapTable T;
  T.keys = static_cast<unsigned long long *>(workspace);
  T.cnt = reinterpret_cast<unsigned *>(T.keys + cap);
  T.mask = cap - 1;
  cudaError_t e = cudaMemsetAsync(T.keys, 0xff, cap * 8, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(T.cnt, 0, (cap + 1) * 8, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(overlap, 0, sizeof(int64_t), st);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  if (n_donor_tokens == 0 || n_target_tokens == 0) return SB_OK;
  const bool d64 = donor_dtype == SB_INDEX_I64, t64 = target_dtype == SB_INDEX_I64;
  if (d64 && t64)
    launch_overlap_count<int64_t, int64_t>(donor_tokens, n_donor_tokens, target_tokens, n_target_tokens, T, st);
  else if (d64)
    launch_overlap_count<int64_t, int32_t>(donor_tokens, n_donor_tokens, target_tokens, n_target_tokens, T, st);
  else if (t64)
    launch_overlap_count<int32_t, int64_t>(donor_tokens, n_donor_tokens, target_tokens, n_target_tokens, T, st);
  else
    launch_overlap_count<int32_t, int32_t>(donor_tokens, n_donor_tokens, target_tokens, n_target_tokens, T, st);
  int s = launch_status();
  if (s != SB_OK) return s;
  const unsigned grid = (unsigned)std::min<uint64_t>((cap + 1 + 255) / 256, 1184);
  overlap_sum_kernel<<<grid, 256, 0, st>>>(T, reinterpret_cast<unsigned long long *>(overlap));
  return launch_status();
}

// Brute-force cosine top-k donor search (sm_100a).
//
// The reference (semblend_core/donor_store.py:323-341) computes, per query,
//     sims = E[valid] @ (q / (||q|| + 1e-8));  keep sims >= min_similarity;
//     top fetch_k by similarity
// in fp32 numpy.  Here a batch of queries is searched in three launches:
//
//  1. prep:    normalise each query exactly as the reference does (fp32), keep
//              the fp32 copy for rescoring and a bf16 copy for the tensor
//              cores, and a per-query bound delta_q on |exact - bf16 score|.
//  2. screen:  a persistent, warp-specialised tcgen05 GEMM of the 16-bit query
//              tile (128 queries, resident in shared memory) against streamed
//              256-donor 16-bit tiles (TMA, 128-byte swizzle), fp32
//              accumulators double-buffered in tensor memory.  The 16-bit copy
//              is fp16 (10 mantissa bits; the default for bounded embeddings)
//              or bf16.  Eight epilogue warps each own one query row and half
//              of the tile's columns and keep, without cross-thread exchange,
//              a register top-k of screening scores; a donor becomes a
//              *candidate* (row, screening score) if its screening score is
//              >= max(min_similarity - delta, L - 2 delta), where L is a lower
//              bound on the k-th best screening score A_k, shared by all CTAs
//              through one atomicMax word per query.
//  3. rescore: per query, the exact A_k over all candidates, then exact fp32
//              dot products (double accumulation) of the candidates whose
//              screening score is >= A_k - 2 delta, threshold, and selection
//              of the top k by (score desc, row asc).
// Every true top-k donor passes both filters: its screening score is >= its
// exact score - delta >= the k-th exact score - delta >= A_k - 2 delta >=
// L - 2 delta (the k rows with the best screening scores all have exact
// scores >= A_k - delta), so the result equals the fp32 computation.
//
// delta_q = ||q~|| max||e - e~|| + ||q - q~|| max||e~|| + ||q - q~|| max||e - e~||
//           + dim 2^-23 ||q~|| max||e~||  (Cauchy-Schwarz on the rounding
// residuals plus the fp32 accumulation error); the row maxima come from
// sb_search_prepare_rows.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <cfloat>

#include "common.cuh"
#include "prof.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace sb {
namespace {

constexpr int kBM = 128;             // queries per tile (one TMEM lane each)
constexpr int kBN = 256;             // donors per MMA tile
constexpr int kBK = 64;              // K elements per shared-memory stage (128 B rows)
constexpr int kQBlockBytes = kBM * 128;
constexpr int kEStageBytes = kBN * 128;
constexpr int kThreads = 320;        // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kMaxTilesPerChunk = 32;  // donor tiles per work unit (chosen per launch, <= this)
#ifndef SB_SCREEN_MAX_STAGES
#define SB_SCREEN_MAX_STAGES 3  // 3 measured as fast as 4 (2 is 10 % slower); leaves ~34 KB of an SM for other kernels
#endif
constexpr int kMaxStages = SB_SCREEN_MAX_STAGES;
constexpr int kSmemLimit = 232448;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

struct ScreenParams {
  int nq;
  int k_blocks;
  int n_qtiles;
  int stages;
  int64_t n_rows;
  int64_t n_ntiles;
  int64_t n_units;
  int tiles_per_chunk;
  float thr;
  int cap;
  uint32_t idesc;
  const uint32_t *valid_bits;  // bit j = row j searchable (bits past n_rows are 0)
  int64_t n_valid_words;
  const float *delta;
  int *count;
  int *lower;
  int2 *cand;  // (row, screening score bits)
  int *status;
  unsigned *sched;  // [next unit, CTAs finished] of this launch's scheduler slot
};

// Work units are handed out dynamically: each CTA's producer thread takes the
// next unit index with an atomic add on a per-launch counter pair in device
// memory, so a CTA whose SM was busy at launch (the sharded search's
// all-gather of the previous batch runs beside this kernel) takes fewer units
// instead of finishing last.  A launch uses one of kSchedSlots slots (round
// robin on the host); the last CTA to finish resets it, so up to kSchedSlots
// launches may be in flight on a device at once.
constexpr int kSchedSlots = 64;
__device__ unsigned g_screen_sched[kSchedSlots * 2];

// Optional clock trace of CTA 0 (compiled out unless SB_SCREEN_TRACE): event
// slot x index -> clock64().
#ifndef SB_SCREEN_TRACE
#define SB_SCREEN_TRACE 0
#endif
#if SB_SCREEN_TRACE
constexpr int kTraceLen = 2048;
__device__ long long g_screen_trace[12 * kTraceLen];
#define SB_STRACE(slot, idx)                                                                        \
  do {                                                                                              \
    if (blockIdx.x == 0 && (idx) < kTraceLen) g_screen_trace[(slot) * kTraceLen + (idx)] = clock64(); \
  } while (0)
#else
#define SB_STRACE(slot, idx) do { } while (0)
#endif

template <typename T> struct Half16;
template <> struct Half16<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float to(__nv_bfloat16 x) { return __bfloat162float(x); }
};
template <> struct Half16<__half> {
  static __device__ __forceinline__ __half from(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float to(__half x) { return __half2float(x); }
};

// Bit-pack the row validity of word w (all rows valid when `valid` is null);
// bits at or past n_rows are cleared.
__device__ __forceinline__ void valid_bits_word(const uint8_t *__restrict__ valid, int64_t n_rows,
                                                uint32_t *__restrict__ bits, int64_t w) {
  uint32_t v = 0;
  const int64_t j0 = w * 32;
  if (valid != nullptr && j0 + 32 <= n_rows && (reinterpret_cast<uintptr_t>(valid) % 16) == 0) {
    const uint4 *p = reinterpret_cast<const uint4 *>(valid + j0);
    const uint4 a = __ldg(p), b = __ldg(p + 1);
    const uint32_t wd[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 32; ++i) v |= (((wd[i / 4] >> (8 * (i % 4))) & 0xffu) != 0 ? 1u : 0u) << i;
  } else {
    for (int i = 0; i < 32; ++i) {
      const int64_t j = j0 + i;
      if (j < n_rows && (valid == nullptr || valid[j])) v |= 1u << i;
    }
  }
  bits[w] = v;
}

template <typename T>
__global__ void query_prep_kernel(const float *__restrict__ q, int64_t ld_q, int nq, int dim, int dim_pad,
                                  const float *__restrict__ stats, float *__restrict__ qn, T *__restrict__ qb,
                                  float *__restrict__ delta, int *__restrict__ count, int *__restrict__ lower,
                                  int q_blocks, const uint8_t *__restrict__ valid, int64_t n_rows,
                                  uint32_t *__restrict__ bits, int64_t n_words) {
  pdl_wait();  // the previous search on this stream still reads this workspace
  pdl_launch_dependents();
  if ((int)blockIdx.x >= q_blocks) {  // trailing blocks: the row-validity bitmask
    const int64_t w = (int64_t)(blockIdx.x - q_blocks) * blockDim.x + threadIdx.x;
    if (w < n_words) valid_bits_word(valid, n_rows, bits, w);
    return;
  }
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= nq) return;
  const float *row = q + (int64_t)warp * ld_q;
  float ss = 0.f;
  for (int i = lane; i < dim; i += 32) ss = fmaf(row[i], row[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  // donor_store.py:326: q / (np.linalg.norm(q) + 1e-8), all in fp32
  const float denom = __fadd_rn(sqrtf(ss), 1e-8f);
  float nb = 0.f, nd = 0.f;
  for (int i = lane; i < dim_pad; i += 32) {
    float v = 0.f;
    if (i < dim) {
      v = __fdiv_rn(row[i], denom);
      qn[(int64_t)warp * dim + i] = v;
    }
    const T b = Half16<T>::from(v);
    qb[(int64_t)warp * dim_pad + i] = b;
    const float bf = Half16<T>::to(b);
    nb = fmaf(bf, bf, nb);
    nd = fmaf(v - bf, v - bf, nd);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nb += __shfl_xor_sync(0xffffffffu, nb, o);
    nd += __shfl_xor_sync(0xffffffffu, nd, o);
  }
  if (lane == 0) {
    const float dmax = stats[0], emax = stats[1];
    const float qbn = sqrtf(nb), dqn = sqrtf(nd);
    const float acc = (float)dim * 1.1920929e-7f * qbn * emax;
    const float d = (qbn * dmax + dqn * emax + dqn * dmax + acc) * 1.001f + 1e-6f;
    delta[warp] = isfinite(d) ? d : INFINITY;  // a 16-bit overflow disables screening
    count[warp] = 0;
    lower[warp] = tc::float_to_ordered(-INFINITY);
  }
}

// Descending insertion into a register-resident sorted list.
template <int KT>
__device__ __forceinline__ void topk_insert(float (&tk)[KT], float s) {
#pragma unroll
  for (int i = KT - 1; i > 0; --i) {
    const float a = tk[i - 1];
    tk[i] = s > a ? a : (s > tk[i] ? s : tk[i]);
  }
  tk[0] = fmaxf(tk[0], s);
}

template <int KT>
__global__ void __launch_bounds__(kThreads, 1)
    screen_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmE,
                  const ScreenParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sE = sQ + P.k_blocks * kQBlockBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sE + P.stages * kEStageBytes);
  uint64_t *full = bars;                   // [kMaxStages]
  uint64_t *empty = bars + kMaxStages;     // [kMaxStages]
  uint64_t *q_full = bars + 2 * kMaxStages;
  uint64_t *q_empty = q_full + 1;
  uint64_t *acc_full = q_full + 2;         // [2]
  uint64_t *acc_empty = q_full + 4;        // [2]
  uint64_t *final_bar = q_full + 6;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(q_full + 7);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(q_full + 8);
  uint64_t *unit_full = q_full + 9;        // [2] unit ring: producer -> MMA thread + epilogue warps
  uint64_t *unit_empty = q_full + 11;      // [2]
  volatile int64_t *unit_ring = reinterpret_cast<volatile int64_t *>(q_full + 13);  // [2]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_empty, 1);
    tc::mbar_init(&acc_full[0], 1);
    tc::mbar_init(&acc_full[1], 1);
    tc::mbar_init(&acc_empty[0], 8);
    tc::mbar_init(&acc_empty[1], 8);
    tc::mbar_init(final_bar, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&unit_full[i], 1);
      tc::mbar_init(&unit_empty[i], 1 + 8);  // the MMA thread and the 8 epilogue warps
    }
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
  pdl_wait();  // query preparation (the previous kernel) has finished and is visible
  if (threadIdx.x == 0) SB_STRACE(9, 0);
  // n-th unit of this CTA (-1: no more work).  A whole warp (epilogue) reads
  // the slot before lane 0 releases it; the single MMA thread releases it itself.
  auto pop_unit = [&](uint32_t n, bool whole_warp) -> int64_t {
    if (!tc::mbar_wait(&unit_full[n & 1], (n >> 1) & 1, ab, 5, kWaitCycles)) return -1;
    const int64_t u = unit_ring[n & 1];
    if (whole_warp) __syncwarp();
    if (!whole_warp || (threadIdx.x & 31) == 0) tc::mbar_arrive(&unit_empty[n & 1]);
    return u;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tc::tma_prefetch_desc(&tmQ);
      tc::tma_prefetch_desc(&tmE);
      uint32_t it = 0, qi = 0, pushed = 0;
      bool ok = true;
      auto push_unit = [&](int64_t u) -> bool {
        const uint32_t slot = pushed & 1, use = pushed >> 1;
        if (use > 0 && !tc::mbar_wait(&unit_empty[slot], (use - 1) & 1, ab, 2, kWaitCycles)) return false;
        unit_ring[slot] = u;
        tc::mbar_arrive(&unit_full[slot]);
        ++pushed;
        return true;
      };
      while (ok) {
        const int64_t u = (int64_t)atomicAdd(P.sched, 1u);
        if (u >= P.n_units) break;
        if (!push_unit(u)) {
          ok = false;
          break;
        }
        const int qt = (int)(u % P.n_qtiles);
        const int64_t t0 = (u / P.n_qtiles) * P.tiles_per_chunk;
        const int64_t t1 = min(t0 + P.tiles_per_chunk, P.n_ntiles);
        if (qi > 0 && !tc::mbar_wait(q_empty, (qi - 1) & 1, ab, 2, kWaitCycles)) break;
        SB_STRACE(5, qi);
        tc::mbar_arrive_expect_tx(q_full, P.k_blocks * kQBlockBytes);
        for (int kb = 0; kb < P.k_blocks; ++kb)
          tc::tma_load_2d(sQ + kb * kQBlockBytes, &tmQ, q_full, kb * kBK, qt * kBM);
        ++qi;
        for (int64_t t = t0; t < t1 && ok; ++t) {
          for (int kb = 0; kb < P.k_blocks; ++kb) {
            const uint32_t s = it % P.stages, ph = (it / P.stages) & 1;
            if (!tc::mbar_wait(&empty[s], ph ^ 1, ab, 2, kWaitCycles)) {
              ok = false;
              break;
            }
            SB_STRACE(4, it);
            tc::mbar_arrive_expect_tx(&full[s], kEStageBytes);
            tc::tma_load_2d(sE + s * kEStageBytes, &tmE, &full[s], kb * kBK, (int)(t * kBN));
            ++it;
          }
        }
      }
      if (ok) push_unit(-1);
      // Let every load this thread issued land before the CTA can exit.
      const uint32_t n_out = it < (uint32_t)P.stages ? it : (uint32_t)P.stages;
      for (uint32_t i = it - n_out; i < it; ++i) {
        const tc::Abort quiet{abort_flag, nullptr};
        volatile int never = 0;
        const tc::Abort drain{&never, nullptr};
        (void)quiet;
        tc::mbar_wait(&full[i % P.stages], (i / P.stages) & 1, drain, 0, kWaitCycles);
      }
      if (qi > 0) {
        volatile int never = 0;
        const tc::Abort drain{&never, nullptr};
        tc::mbar_wait(q_full, (qi - 1) & 1, drain, 0, kWaitCycles);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = P.idesc;
      uint32_t it = 0, qi = 0, ai = 0;
      bool ok = true;
      for (uint32_t n = 0; ok; ++n) {
        const int64_t u = pop_unit(n, false);
        if (u < 0) break;
        const int64_t t0 = (u / P.n_qtiles) * P.tiles_per_chunk;
        const int64_t t1 = min(t0 + P.tiles_per_chunk, P.n_ntiles);
        if (!tc::mbar_wait(q_full, qi & 1, ab, 3, kWaitCycles)) break;
        SB_STRACE(3, qi);
        tc::fence_after_sync();
        for (int64_t t = t0; t < t1 && ok; ++t) {
          const uint32_t b = ai & 1;
          if (!tc::mbar_wait(&acc_empty[b], ((ai >> 1) & 1) ^ 1, ab, 3, kWaitCycles)) {
            ok = false;
            break;
          }
          SB_STRACE(2, ai);
          tc::fence_after_sync();
          const uint32_t d_tmem = tmem + b * kBN;
          for (int kb = 0; kb < P.k_blocks; ++kb) {
            const uint32_t s = it % P.stages, ph = (it / P.stages) & 1;
            if (!tc::mbar_wait(&full[s], ph, ab, 3, kWaitCycles)) {
              ok = false;
              break;
            }
            SB_STRACE(0, it);
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t da = tc::desc_kmajor_sw128(sQ + kb * kQBlockBytes, kk * 32);
              const uint64_t db = tc::desc_kmajor_sw128(sE + s * kEStageBytes, kk * 32);
              tc::mma_bf16_ss(d_tmem, da, db, idesc, (kb | kk) != 0);
            }
            tc::mma_commit(&empty[s]);
            SB_STRACE(1, it);
            ++it;
          }
          if (!ok) break;
          tc::mma_commit(&acc_full[b]);
          ++ai;
        }
        tc::mma_commit(q_empty);
        ++qi;
      }
      // All MMAs this thread issued must finish before TMEM is released.
      tc::mma_commit(final_bar);
      volatile int never = 0;
      const tc::Abort drain{&never, nullptr};
      tc::mbar_wait(final_bar, 0, drain, 0, kWaitCycles);
    }
  } else {
    // ---------------- epilogue ----------------
    // 8 warps: warp w reads TMEM lanes [32*(w%4), +32) (its quarter of the
    // query rows) and one half of the tile's 256 donor columns, so every
    // query row is scanned by two threads, each with its own top-k list.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    uint32_t ai = 0;
    bool ok = true;
    for (uint32_t n = 0; ok; ++n) {
      const int64_t u = pop_unit(n, true);
      if (u < 0) break;
      const int qt = (int)(u % P.n_qtiles);
      const int64_t t0 = (u / P.n_qtiles) * P.tiles_per_chunk;
      const int64_t t1 = min(t0 + P.tiles_per_chunk, P.n_ntiles);
      const int q = qt * kBM + row;
      const bool active = q < P.nq;
      const float dq = active ? P.delta[q] : 0.f;
      const float two_d = 2.f * dq;
      float tk[KT];
#pragma unroll
      for (int i = 0; i < KT; ++i) tk[i] = -INFINITY;
      float cut = P.thr - dq;
      for (int64_t t = t0; t < t1; ++t) {
        const int64_t c0 = t * kBN + half * (kBN / 2);  // first donor column of this thread
        // prefetch: validity bits of the 128 columns and the shared lower bound
        uint32_t vb[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int64_t word = (c0 >> 5) + w;
          vb[w] = word < P.n_valid_words ? __ldg(P.valid_bits + word) : 0u;
        }
        const int lg = active ? *reinterpret_cast<volatile int *>(P.lower + q) : 0;
        const uint32_t b = ai & 1;
        if (!tc::mbar_wait(&acc_full[b], (ai >> 1) & 1, ab, 4, kWaitCycles)) {
          ok = false;
          break;
        }
        if (warp == 2 && lane == 0) SB_STRACE(6, ai);
        tc::fence_after_sync();
        const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + b * kBN + half * (kBN / 2);
        const float tk_before = tk[KT - 1];
        int nc = 0;
        int2 cb0 = make_int2(0, 0), cb1 = cb0, cb2 = cb0, cb3 = cb0;
#pragma unroll 1
        for (int c = 0; c < kBN / 2; c += 64) {
          uint32_t r0[32], r1[32];
          tc::tmem_ld32(base + c, r0);
          tc::tmem_ld32(base + c + 32, r1);
          tc::tmem_ld_wait();
          if (!active) continue;
          // hot path: the 64 columns' maximum (NaN-propagating 3-input max, ~0.5
          // instruction per column) against the cut; almost every group ends here
          {
            float a[22];
#pragma unroll
            for (int i = 0; i < 10; ++i)
              a[i] = tc::max3_nan(__uint_as_float(r0[3 * i]), __uint_as_float(r0[3 * i + 1]),
                                  __uint_as_float(r0[3 * i + 2]));
            a[10] = tc::max3_nan(__uint_as_float(r0[30]), __uint_as_float(r0[31]), __uint_as_float(r1[0]));
#pragma unroll
            for (int i = 0; i < 10; ++i)
              a[11 + i] = tc::max3_nan(__uint_as_float(r1[3 * i + 1]), __uint_as_float(r1[3 * i + 2]),
                                       __uint_as_float(r1[3 * i + 3]));
            a[21] = __uint_as_float(r1[31]);
#pragma unroll
            for (int i = 0; i < 7; ++i) a[i] = tc::max3_nan(a[3 * i], a[3 * i + 1], a[3 * i + 2]);
            a[7] = a[21];  // a[0..7]: 8 partial maxima
            const float mx = tc::max3_nan(tc::max3_nan(a[0], a[1], a[2]), tc::max3_nan(a[3], a[4], a[5]),
                                          tc::max3_nan(a[6], a[7], a[7]));
            if (mx < cut) continue;  // false for NaN: such groups take the exact path below
          }
          // one compare per column into a hit mask
          // (!(x < cut) also keeps NaN scores, and everything once cut is -inf)
          uint32_t h0 = 0, h1 = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            h0 |= (__uint_as_float(r0[i]) < cut ? 0u : 1u) << i;
            h1 |= (__uint_as_float(r1[i]) < cut ? 0u : 1u) << i;
          }
          h0 &= vb[c >> 5];
          h1 &= vb[(c >> 5) + 1];
          // rare path, emitted once: every hit becomes a candidate
#pragma unroll 1
          while (h0 | h1) {
            const bool lo = h0 != 0;
            const int i = __ffs(lo ? h0 : h1) - 1;
            if (lo) h0 &= h0 - 1; else h1 &= h1 - 1;
            uint32_t bits = 0;
#pragma unroll
            for (int x = 0; x < 32; ++x) bits = (x == i) ? (lo ? r0[x] : r1[x]) : bits;
            const float sc = __uint_as_float(bits);
            const int2 e = make_int2((int)(c0 + c + (lo ? 0 : 32) + i), (int)bits);
            if (nc == 0) cb0 = e;
            else if (nc == 1) cb1 = e;
            else if (nc == 2) cb2 = e;
            else cb3 = e;
            if (++nc == 4) {
              const int slot = atomicAdd(&P.count[q], 4);
              int2 *dst = P.cand + (int64_t)q * P.cap;
              if (slot + 0 < P.cap) dst[slot + 0] = cb0;
              if (slot + 1 < P.cap) dst[slot + 1] = cb1;
              if (slot + 2 < P.cap) dst[slot + 2] = cb2;
              if (slot + 3 < P.cap) dst[slot + 3] = cb3;
              nc = 0;
            }
            if (sc > tk[KT - 1]) {
              topk_insert<KT>(tk, sc);
              cut = fmaxf(cut, tk[KT - 1] - two_d);
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
        if (warp == 2 && lane == 0) SB_STRACE(7, ai);
        if (warp == 9 && lane == 0) SB_STRACE(8, ai);
        ++ai;
        if (active) {
          if (nc) {
            const int slot = atomicAdd(&P.count[q], nc);
            int2 *dst = P.cand + (int64_t)q * P.cap;
            if (slot + 0 < P.cap) dst[slot + 0] = cb0;
            if (nc > 1 && slot + 1 < P.cap) dst[slot + 1] = cb1;
            if (nc > 2 && slot + 2 < P.cap) dst[slot + 2] = cb2;
          }
          if (tk[KT - 1] > tk_before) atomicMax(&P.lower[q], tc::float_to_ordered(tk[KT - 1]));
          cut = fmaxf(cut, tc::ordered_to_float(lg) - two_d);
        }
      }
    }
  }

  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0) {
    // every producer of this launch has stopped taking units once all CTAs got here
    __threadfence();
    if (atomicAdd(P.sched + 1, 1u) == gridDim.x - 1) {
      P.sched[0] = 0;
      P.sched[1] = 0;
      __threadfence();
    }
  }
}

// Per query (one warp each): the exact k-th best screening score A_k over the
// candidates, exact rescoring (fp64 accumulation of the fp32 vectors) of the
// candidates with screening score >= A_k - 2 delta, threshold and top-k
// selection by (score desc, row asc).
//
// The kernel is latency-bound (a query rescored ~10-30 rows here), so every
// stage keeps several loads in flight per lane.  A_k: every lane keeps a
// sorted register list of the best KT screening scores of its strided share
// of the candidates (read 8 per lane at a time); k rounds of a warp max over
// the list heads pop the k best.  Candidates that pass the A_k filter are
// queued in shared memory and rescored a few rows at a time, each row split
// over the warp (T 16-byte loads per lane per row, T = ceil(dim / 128)), all
// loads of those rows in flight together.  The result list is spread over
// the warp: lane j holds the j-th best (score, row) so far, and an insertion
// is one ballot plus one shuffle.
constexpr int kRescoreWarps = 8;
constexpr int kMaxDim = 512;
constexpr int kCandPerLane = 8;                 // candidates read per lane and pass
constexpr int kQueue = 32 * kCandPerLane + 32;  // passing candidates queued per warp

__device__ __forceinline__ bool better(float s, int id, float s2, int id2) {
  return s > s2 || (s == s2 && id < id2);
}

template <int KT, int T>
__global__ void __launch_bounds__(kRescoreWarps * 32, 4)
    rescore_kernel(const float *__restrict__ emb, int64_t ld_emb, int dim, const float *__restrict__ qn,
                   const float *__restrict__ delta, const int *__restrict__ count, const int2 *__restrict__ cand,
                   int cap, float thr, int k, int nq, int64_t id_offset, int64_t *__restrict__ out_ids,
                   float *__restrict__ out_scores, int *status) {
  __shared__ __align__(16) float sq_all[kRescoreWarps][kMaxDim];
  __shared__ int queue_all[kRescoreWarps][kQueue];
  pdl_wait();  // the screening kernel's candidates are complete and visible
  pdl_launch_dependents();
  const int lane = threadIdx.x % 32, wib = threadIdx.x / 32;
  const int q = blockIdx.x * kRescoreWarps + wib;
  if (q >= nq) return;
  float *qv = sq_all[wib];
  int *queue = queue_all[wib];
  int n = count[q];
  if (n > cap) {
    if (lane == 0) atomicOr(status, 1);
    n = 0;  // results for this query are withheld (reported as overflow)
  }
  const int2 *cq = cand + (int64_t)q * cap;
  const int *cq_score = reinterpret_cast<const int *>(cq) + 1;  // .y of each entry
  for (int d = lane; d < dim; d += 32) qv[d] = qn[(int64_t)q * dim + d];

  float keep = -INFINITY;  // screening-score floor for exact rescoring
  if (n > k) {
    float tk[KT];
#pragma unroll
    for (int i = 0; i < KT; ++i) tk[i] = -INFINITY;
    for (int base = 0; base < n; base += 32 * kCandPerLane) {
      float v[kCandPerLane];
#pragma unroll
      for (int j = 0; j < kCandPerLane; ++j) {
        const int i = base + 32 * j + lane;
        v[j] = i < n ? __int_as_float(__ldcg(cq_score + 2 * (int64_t)i)) : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < kCandPerLane; ++j)
        if (v[j] > tk[KT - 1]) topk_insert<KT>(tk, v[j]);  // NaN never enters
    }
    int popped = INT_MIN;
    for (int r = 0; r < k; ++r) {
      const int head = tc::float_to_ordered(tk[0]);
      popped = __reduce_max_sync(0xffffffffu, head);
      const uint32_t holders = __ballot_sync(0xffffffffu, head == popped);
      if (lane == __ffs(holders) - 1) {
#pragma unroll
        for (int i = 0; i < KT - 1; ++i) tk[i] = tk[i + 1];
        tk[KT - 1] = -INFINITY;
      }
    }
    const float ak = tc::ordered_to_float(popped);  // -inf if fewer than k finite scores
    const float dq = delta[q];
    keep = isfinite(dq) ? ak - 2.f * dq : -INFINITY;
  }
  __syncwarp();

  // warp-spread result list: lane j < k holds the j-th best so far
  float ls = -INFINITY;
  int li = INT_MAX;
  const bool vec4 = (dim % 4 == 0) && (ld_emb % 4 == 0) && (reinterpret_cast<uintptr_t>(emb) % 16 == 0);
  const float4 *qv4 = reinterpret_cast<const float4 *>(qv);

  // insert (s, id) (warp-uniform) into the list
  auto insert = [&](float ns, int ni) {
    if (!(ns >= thr) || ns == -INFINITY) return;
    const uint32_t ahead = __ballot_sync(0xffffffffu, lane < k && better(ls, li, ns, ni));
    const int pos = __popc(ahead);
    const float us = __shfl_up_sync(0xffffffffu, ls, 1);
    const int ui = __shfl_up_sync(0xffffffffu, li, 1);
    if (pos < k) {
      if (lane > pos) ls = us, li = ui;
      if (lane == pos) ls = ns, li = ni;
    }
  };

  // exact scores of the rows queue[off, off + cnt): the warp splits each row's
  // dims (16 bytes per lane), ROWS rows with all their loads in flight at once
  auto flush = [&](int off, int cnt) {
    constexpr int ROWS = T <= 2 ? 4 : 2;
    for (int r0 = 0; r0 < cnt; r0 += ROWS) {
      int id[ROWS];
      double acc[ROWS];
      float4 v[ROWS][T];
#pragma unroll
      for (int j = 0; j < ROWS; ++j) {
        id[j] = r0 + j < cnt ? queue[off + r0 + j] : -1;
        const float *row = emb + (int64_t)max(id[j], 0) * ld_emb;
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int c = lane + 32 * t;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (id[j] >= 0 && 4 * c < dim) {
            if (vec4) {
              x = __ldg(reinterpret_cast<const float4 *>(row) + c);
            } else {  // rows not 16-byte aligned: element loads
              x.x = __ldg(row + 4 * c);
              if (4 * c + 1 < dim) x.y = __ldg(row + 4 * c + 1);
              if (4 * c + 2 < dim) x.z = __ldg(row + 4 * c + 2);
              if (4 * c + 3 < dim) x.w = __ldg(row + 4 * c + 3);
            }
          }
          v[j][t] = x;
        }
      }
#pragma unroll
      for (int j = 0; j < ROWS; ++j) {
        double a = 0.0;
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int c = lane + 32 * t;
          const float4 w = 4 * c < dim ? qv4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
          a = fma((double)w.x, (double)v[j][t].x, a);
          a = fma((double)w.y, (double)v[j][t].y, a);
          a = fma((double)w.z, (double)v[j][t].z, a);
          a = fma((double)w.w, (double)v[j][t].w, a);
        }
        acc[j] = a;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < ROWS; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (id[j] >= 0) insert((float)acc[j], id[j]);
    }
  };

  int queued = 0;  // warp-uniform, < 32 between passes
  for (int base = 0;; base += 32 * kCandPerLane) {
    const bool last = base + 32 * kCandPerLane >= n;
    if (base < n) {
      int2 e[kCandPerLane];
#pragma unroll
      for (int j = 0; j < kCandPerLane; ++j) {
        const int i = base + 32 * j + lane;
        e[j] = i < n ? __ldcg(cq + i) : make_int2(0, 0);
      }
#pragma unroll
      for (int j = 0; j < kCandPerLane; ++j) {
        const int i = base + 32 * j + lane;
        const bool pass = i < n && !(__int_as_float(e[j].y) < keep);  // NaN screening scores are always rescored
        const uint32_t m = __ballot_sync(0xffffffffu, pass);
        if (pass) queue[queued + __popc(m & ((1u << lane) - 1))] = e[j].x;
        queued += __popc(m);
      }
      __syncwarp();
    }
    // full batches now; the remainder after the last pass
    int off = 0;
    while (queued - off >= 32 || (last && queued - off > 0)) {
      const int cnt = min(32, queued - off);
      flush(off, cnt);
      off += cnt;
    }
    if (last) break;
    const int rest = queued - off;  // < 32: move to the front
    const int moved = lane < rest ? queue[off + lane] : 0;
    __syncwarp();
    if (lane < rest) queue[lane] = moved;
    __syncwarp();
    queued = rest;
  }
  if (lane < k) {
    const bool hit = ls > -INFINITY;
    out_ids[(int64_t)q * k + lane] = hit ? (int64_t)li + id_offset : -1;
    out_scores[(int64_t)q * k + lane] = hit ? ls : -INFINITY;
  }
}

__global__ void fill_empty_kernel(int64_t *ids, float *scores, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) ids[i] = -1, scores[i] = -INFINITY;
}

template <typename T>
__global__ void prepare_rows_kernel(const float *__restrict__ emb, int64_t ld_emb, T *__restrict__ eb, int64_t ld_b,
                                    int dim, int dim_pad, const int64_t *__restrict__ rows, int64_t row_begin,
                                    int64_t n, float *stats) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= n) return;
  const int64_t r = rows != nullptr ? rows[w] : row_begin + w;
  const float *e = emb + r * ld_emb;
  float nb = 0.f, nd = 0.f;
  for (int i = lane; i < dim_pad; i += 32) {
    const float v = i < dim ? e[i] : 0.f;
    const T b = Half16<T>::from(v);
    eb[r * ld_b + i] = b;
    const float bf = Half16<T>::to(b);
    nb = fmaf(bf, bf, nb);
    nd = fmaf(v - bf, v - bf, nd);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nb += __shfl_xor_sync(0xffffffffu, nb, o);
    nd += __shfl_xor_sync(0xffffffffu, nd, o);
  }
  if (lane == 0) {
    // non-negative floats order like their bit patterns; a non-finite norm
    // (a value outside the 16-bit range) poisons the bound to +inf
    const float dn = sqrtf(nd) * 1.0001f, bn = sqrtf(nb) * 1.0001f;
    atomicMax(reinterpret_cast<int *>(&stats[0]), __float_as_int(isfinite(dn) ? dn : INFINITY));
    atomicMax(reinterpret_cast<int *>(&stats[1]), __float_as_int(isfinite(bn) ? bn : INFINITY));
  }
}

// Merge n_lists sorted top-k lists per query (shards of a row-partitioned
// search) into one, by (score desc, id asc).  One warp per query: lane l holds
// list l in registers; k rounds of a warp argmax over the list heads, the
// winning lane shifts its list.
constexpr int kMergeWarps = 8;

template <int KT>
__global__ void __launch_bounds__(kMergeWarps * 32)
    topk_merge_kernel(const int64_t *__restrict__ ids, int64_t ids_stride, const float *__restrict__ scores,
                      int64_t scores_stride, int n_lists, int nq, int k, int64_t *__restrict__ out_ids,
                      float *__restrict__ out_scores) {
  const int lane = threadIdx.x % 32;
  const int q = blockIdx.x * kMergeWarps + threadIdx.x / 32;
  if (q >= nq) return;
  float ls[KT];
  int64_t li[KT];
#pragma unroll
  for (int j = 0; j < KT; ++j) {
    ls[j] = -INFINITY;
    li[j] = -1;
    if (lane < n_lists && j < k) {
      const int64_t off = (int64_t)q * k + j;
      li[j] = ids[lane * ids_stride + off];
      ls[j] = li[j] >= 0 ? scores[lane * scores_stride + off] : -INFINITY;
    }
  }
  for (int r = 0; r < k; ++r) {
    float bs = li[0] >= 0 ? ls[0] : -INFINITY;
    int64_t bi = li[0] >= 0 ? li[0] : INT64_MAX;
    int bl = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
      if (os > bs || (os == bs && (oi < bi || (oi == bi && ol < bl)))) bs = os, bi = oi, bl = ol;
    }
    const bool hit = bi != INT64_MAX;
    if (lane == bl && hit) {
#pragma unroll
      for (int j = 0; j < KT - 1; ++j) ls[j] = ls[j + 1], li[j] = li[j + 1];
      ls[KT - 1] = -INFINITY, li[KT - 1] = -1;
    }
    if (lane == 0) {
      out_ids[(int64_t)q * k + r] = hit ? bi : -1;
      out_scores[(int64_t)q * k + r] = hit ? bs : -INFINITY;
    }
  }
}

template <int KT>
void launch_rescore_kt(int t, unsigned grid, cudaStream_t st, const float *emb, int64_t ld_emb, int dim,
                       const float *qn, const float *delta, const int *count, const int2 *cand, int cap, float thr,
                       int k, int nq, int64_t id_offset, int64_t *out_ids, float *out_scores, int *status) {
  const dim3 block(kRescoreWarps * 32);
  if (t == 1)
    launch_pdl(rescore_kernel<KT, 1>, grid, block, 0, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq,
                                                  id_offset, out_ids, out_scores, status);
  else if (t == 2)
    launch_pdl(rescore_kernel<KT, 2>, grid, block, 0, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq,
                                                  id_offset, out_ids, out_scores, status);
  else if (t == 3)
    launch_pdl(rescore_kernel<KT, 3>, grid, block, 0, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq,
                                                  id_offset, out_ids, out_scores, status);
  else
    launch_pdl(rescore_kernel<KT, 4>, grid, block, 0, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq,
                                                  id_offset, out_ids, out_scores, status);
}

void launch_rescore(int kt, unsigned grid, cudaStream_t st, const float *emb, int64_t ld_emb, int dim,
                    const float *qn, const float *delta, const int *count, const int2 *cand, int cap, float thr,
                    int k, int nq, int64_t id_offset, int64_t *out_ids, float *out_scores, int *status) {
  const int t = (dim + 127) / 128;  // 16-byte loads per lane per row (dim <= 512)
  if (kt == 8)
    launch_rescore_kt<8>(t, grid, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq, id_offset, out_ids,
                         out_scores, status);
  else if (kt == 16)
    launch_rescore_kt<16>(t, grid, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq, id_offset,
                          out_ids, out_scores, status);
  else
    launch_rescore_kt<32>(t, grid, st, emb, ld_emb, dim, qn, delta, count, cand, cap, thr, k, nq, id_offset,
                          out_ids, out_scores, status);
}

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct Workspace {
  int *count, *lower;
  float *delta, *qn;
  void *qb;
  int2 *cand;
  uint32_t *bits;
  int64_t bytes;
};

Workspace carve(void *base, int nq, int dim, int dim_pad, int cap, int64_t n_rows) {
  Workspace w;
  char *p = reinterpret_cast<char *>(base);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char *r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  w.count = reinterpret_cast<int *>(take(4LL * nq));
  w.lower = reinterpret_cast<int *>(take(4LL * nq));
  w.delta = reinterpret_cast<float *>(take(4LL * nq));
  w.qn = reinterpret_cast<float *>(take(4LL * nq * dim));
  w.qb = take(2LL * nq * dim_pad);
  w.cand = reinterpret_cast<int2 *>(take(8LL * nq * cap));
  w.bits = reinterpret_cast<uint32_t *>(take(4LL * ((n_rows + 31) / 32 + 8)));
  w.bytes = off;
  return w;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

// This launch's scheduler counter pair on the current device (the symbol's
// address is looked up once per device, with that device current).
unsigned *screen_sched_slot() {
  static std::mutex mu;
  static unsigned *base[64] = {};
  static std::atomic<unsigned> next{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_cuda_error(e);
    return nullptr;
  }
  {
    std::lock_guard<std::mutex> lock(mu);
    if (base[dev] == nullptr) {
      void *p = nullptr;
      e = cudaGetSymbolAddress(&p, g_screen_sched);
      if (e != cudaSuccess || p == nullptr) {
        set_last_cuda_error(e);
        return nullptr;
      }
      base[dev] = static_cast<unsigned *>(p);
    }
  }
  return base[dev] + 2 * (next.fetch_add(1) % kSchedSlots);
}

template <int KT>
int launch_screen(const CUtensorMap &tq, const CUtensorMap &te, const ScreenParams &P, int grid, int smem,
                  cudaStream_t st) {
  if (ensure_dynamic_smem(reinterpret_cast<const void *>(screen_kernel<KT>), smem) != SB_OK) return SB_ERR_CUDA;
  const int slot = prof_before(st);
  const cudaError_t e = launch_pdl(screen_kernel<KT>, dim3(grid), dim3(kThreads), smem, st, tq, te, P);
  prof_after(slot, st);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  return launch_status();
}

}  // namespace
}  // namespace sb

#if SB_SCREEN_TRACE
extern "C" SB_API int sb_screen_trace_read(long long *dst) {
  return cudaMemcpyFromSymbol(dst, sb::g_screen_trace, sizeof(sb::g_screen_trace)) == cudaSuccess ? 0 : -3;
}
extern "C" SB_API int sb_screen_trace_reset() {
  void *p = nullptr;
  if (cudaGetSymbolAddress(&p, sb::g_screen_trace) != cudaSuccess) return -3;
  return cudaMemset(p, 0, sizeof(sb::g_screen_trace)) == cudaSuccess ? 0 : -3;
}
#endif

extern "C" SB_API int sb_search_prepare_rows(const float *emb, int64_t ld_emb, void *emb16, int64_t ld_16,
                                             int32_t dim, int32_t dim_pad, int32_t shadow_dtype, const int64_t *rows,
                                             int64_t row_begin, int64_t n_rows, float *stats, void *stream) {
  if (n_rows < 0 || dim <= 0 || dim_pad < dim || ld_emb < dim || ld_16 < dim_pad) return SB_ERR_INVALID_ARGUMENT;
  if (shadow_dtype != SB_DTYPE_F16 && shadow_dtype != SB_DTYPE_BF16) return SB_ERR_UNSUPPORTED;
  if (n_rows == 0) return SB_OK;
  if (emb == nullptr || emb16 == nullptr || stats == nullptr) return SB_ERR_INVALID_ARGUMENT;
  const int64_t threads = 256, warps_per_block = threads / 32;
  const int64_t blocks = (n_rows + warps_per_block - 1) / warps_per_block;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (shadow_dtype == SB_DTYPE_F16)
    sb::prepare_rows_kernel<__half><<<(unsigned)blocks, (unsigned)threads, 0, st>>>(
        emb, ld_emb, reinterpret_cast<__half *>(emb16), ld_16, dim, dim_pad, rows, row_begin, n_rows, stats);
  else
    sb::prepare_rows_kernel<__nv_bfloat16><<<(unsigned)blocks, (unsigned)threads, 0, st>>>(
        emb, ld_emb, reinterpret_cast<__nv_bfloat16 *>(emb16), ld_16, dim, dim_pad, rows, row_begin, n_rows, stats);
  return sb::launch_status();
}

extern "C" SB_API int64_t sb_cosine_topk_workspace_bytes(int32_t n_queries, int64_t n_rows, int32_t dim,
                                                         int32_t dim_pad, int32_t capacity) {
  if (n_queries < 0 || n_rows < 0 || dim <= 0 || dim_pad < dim || capacity <= 0) return -1;
  return sb::carve(nullptr, n_queries, dim, dim_pad, capacity, n_rows).bytes;
}

namespace sb {
namespace {

// Argument checks shared by the screening and rescoring phases.
int check_topk_args(int64_t ld_emb, int64_t n_rows, int32_t dim, int32_t dim_pad, int32_t n_queries, int32_t k,
                    int32_t capacity, const int64_t *out_ids, const float *out_scores, const int32_t *status) {
  if (n_queries < 0 || n_rows < 0 || k < 1 || k > 32 || dim <= 0) return SB_ERR_INVALID_ARGUMENT;
  if (dim_pad < dim || dim_pad % kBK != 0 || dim_pad > 512) return SB_ERR_UNSUPPORTED;
  if (capacity < k || capacity > 16384) return SB_ERR_INVALID_ARGUMENT;
  if (n_rows > 0x7fffffffLL) return SB_ERR_TOO_LARGE;
  if (n_queries == 0) return SB_OK;
  if (ld_emb < dim || status == nullptr || (out_ids == nullptr) != (out_scores == nullptr))
    return SB_ERR_INVALID_ARGUMENT;
  return SB_OK;
}

// Query preparation and the tensor-core screening kernel: each query's
// candidates with their screening scores and its error bound, into the
// workspace.
int cosine_screen(const void *emb16, int64_t ld_16, int32_t shadow_dtype, const uint8_t *valid, int64_t n_rows,
                  int32_t dim, int32_t dim_pad, const float *stats, const float *queries, int64_t ld_q,
                  int32_t n_queries, int32_t k, float min_similarity, int32_t capacity, const Workspace &w,
                  int32_t *status, cudaStream_t st) {
  const bool f16 = shadow_dtype == SB_DTYPE_F16;
  const int64_t n_words = (n_rows + 31) / 32;
  {
    const int threads = 256;
    const int q_blocks = (n_queries * 32 + threads - 1) / threads;
    const int blocks = q_blocks + (int)((n_words + threads - 1) / threads);
    if (f16)
      query_prep_kernel<__half><<<blocks, threads, 0, st>>>(queries, ld_q, n_queries, dim, dim_pad, stats, w.qn,
                                                            reinterpret_cast<__half *>(w.qb), w.delta, w.count,
                                                            w.lower, q_blocks, valid, n_rows, w.bits, n_words);
    else
      query_prep_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
          queries, ld_q, n_queries, dim, dim_pad, stats, w.qn, reinterpret_cast<__nv_bfloat16 *>(w.qb), w.delta,
          w.count, w.lower, q_blocks, valid, n_rows, w.bits, n_words);
    int s = launch_status();
    if (s != SB_OK) return s;
  }

  CUtensorMap tq, te;
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap_16_2d(&tq, dt, w.qb, dim_pad, n_queries, (uint64_t)dim_pad * 2, kBK, kBM) ||
      !make_tmap_16_2d(&te, dt, emb16, dim_pad, n_rows, (uint64_t)ld_16 * 2, kBK, kBN))
    return SB_ERR_CUDA;

  ScreenParams P;
  P.nq = n_queries;
  P.k_blocks = dim_pad / kBK;
  P.n_qtiles = (n_queries + kBM - 1) / kBM;
  P.n_rows = n_rows;
  P.n_ntiles = (n_rows + kBN - 1) / kBN;
  // Work unit = one query tile x a chunk of donor tiles; the query tiles of a
  // chunk are consecutive units, so concurrent CTAs share each chunk through
  // L2.  The chunk length balances the last wave of units across the SMs
  // (one tile-equivalent charged per unit for its query-tile load).
  {
    const int sms = sm_count();
    int64_t best_cost = INT64_MAX;
    for (int tpc = kMaxTilesPerChunk; tpc >= 8; tpc /= 2) {
      const int64_t units = (P.n_ntiles + tpc - 1) / tpc * P.n_qtiles;
      const int64_t g = std::min<int64_t>(sms, units);
      const int64_t cost = (units + g - 1) / g * (tpc + 1);
      if (cost < best_cost) best_cost = cost, P.tiles_per_chunk = tpc, P.n_units = units;
    }
  }
  P.thr = min_similarity;
  P.cap = capacity;
  P.idesc = tc::idesc_f16(kBM, kBN, f16 ? 0u : 1u, 0u);
  P.valid_bits = w.bits;
  P.n_valid_words = n_words;
  P.delta = w.delta;
  P.count = w.count;
  P.lower = w.lower;
  P.cand = w.cand;
  P.status = status;
  const int fixed = 1024 + P.k_blocks * kQBlockBytes + 256;
  P.stages = std::min<int>(kMaxStages, (kSmemLimit - fixed) / kEStageBytes);
  if (P.stages < 2) return SB_ERR_UNSUPPORTED;
  const int smem = fixed + P.stages * kEStageBytes;
  const int grid = (int)std::min<int64_t>(sm_count(), P.n_units);
  P.sched = screen_sched_slot();
  if (P.sched == nullptr) return SB_ERR_CUDA;
  int s;
  if (k <= 8)
    s = launch_screen<8>(tq, te, P, grid, smem, st);
  else if (k <= 16)
    s = launch_screen<16>(tq, te, P, grid, smem, st);
  else
    s = launch_screen<32>(tq, te, P, grid, smem, st);
  return s;
}

// Exact rescoring of the screened candidates and top-k selection.
int cosine_rescore(const float *emb, int64_t ld_emb, int64_t n_rows, int32_t dim, int32_t n_queries, int32_t k,
                   float min_similarity, int64_t id_offset, int64_t *out_ids, float *out_scores, int32_t capacity,
                   const Workspace &w, int32_t *status, cudaStream_t st) {
  if (n_rows == 0) {
    const int64_t n = (int64_t)n_queries * k;
    fill_empty_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(out_ids, out_scores, n);
    return launch_status();
  }
  const unsigned rs_grid = (unsigned)((n_queries + kRescoreWarps - 1) / kRescoreWarps);
  const int kt = k <= 8 ? 8 : (k <= 16 ? 16 : 32);
  launch_rescore(kt, rs_grid, st, emb, ld_emb, dim, w.qn, w.delta, w.count, w.cand, capacity, min_similarity, k,
                 n_queries, id_offset, out_ids, out_scores, status);
  return launch_status();
}

}  // namespace
}  // namespace sb

extern "C" SB_API int sb_cosine_screen(const void *emb16, int64_t ld_16, int32_t shadow_dtype, const uint8_t *valid,
                                       int64_t n_rows, int32_t dim, int32_t dim_pad, const float *stats,
                                       const float *queries, int64_t ld_q, int32_t n_queries, int32_t k,
                                       float min_similarity, int32_t capacity, void *workspace,
                                       int64_t workspace_bytes, int32_t *status, void *stream) {
  using namespace sb;
  int s = check_topk_args(dim, n_rows, dim, dim_pad, n_queries, k, capacity, nullptr, nullptr, status);
  if (s != SB_OK) return s;
  if (shadow_dtype != SB_DTYPE_F16 && shadow_dtype != SB_DTYPE_BF16) return SB_ERR_UNSUPPORTED;
  if (n_queries == 0) return SB_OK;
  if (n_rows == 0) {
    const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) set_last_cuda_error(e);
    return e == cudaSuccess ? SB_OK : SB_ERR_CUDA;
  }
  if (queries == nullptr || stats == nullptr || emb16 == nullptr) return SB_ERR_INVALID_ARGUMENT;
  if (ld_q < dim || ld_16 < dim_pad) return SB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(emb16) % 16) || ((ld_16 * 2) % 16)) return SB_ERR_INVALID_ARGUMENT;
  const Workspace w = carve(workspace, n_queries, dim, dim_pad, capacity, n_rows);
  if (workspace == nullptr || workspace_bytes < w.bytes) return SB_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  return cosine_screen(emb16, ld_16, shadow_dtype, valid, n_rows, dim, dim_pad, stats, queries, ld_q, n_queries, k,
                       min_similarity, capacity, w, status, st);
}

extern "C" SB_API int sb_cosine_rescore(const float *emb, int64_t ld_emb, int64_t n_rows, int32_t dim,
                                        int32_t dim_pad, int32_t n_queries, int32_t k, float min_similarity,
                                        int64_t id_offset, int64_t *out_ids, float *out_scores, int32_t capacity,
                                        void *workspace, int64_t workspace_bytes, int32_t *status, void *stream) {
  using namespace sb;
  int s = check_topk_args(ld_emb, n_rows, dim, dim_pad, n_queries, k, capacity, out_ids, out_scores, status);
  if (s != SB_OK) return s;
  if (n_queries == 0) return SB_OK;
  if (out_ids == nullptr) return SB_ERR_INVALID_ARGUMENT;
  const Workspace w = carve(workspace, n_queries, dim, dim_pad, capacity, n_rows);
  if (n_rows > 0 && (emb == nullptr || workspace == nullptr || workspace_bytes < w.bytes))
    return emb == nullptr ? SB_ERR_INVALID_ARGUMENT : SB_ERR_WORKSPACE_TOO_SMALL;
  return cosine_rescore(emb, ld_emb, n_rows, dim, n_queries, k, min_similarity, id_offset, out_ids, out_scores,
                        capacity, w, status, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" SB_API int sb_cosine_topk(const float *emb, int64_t ld_emb, const void *emb16, int64_t ld_16,
                                     int32_t shadow_dtype, const uint8_t *valid, int64_t n_rows, int32_t dim,
                                     int32_t dim_pad, const float *stats, const float *queries, int64_t ld_q,
                                     int32_t n_queries, int32_t k, float min_similarity, int64_t id_offset,
                                     int64_t *out_ids, float *out_scores, int32_t capacity, void *workspace,
                                     int64_t workspace_bytes, int32_t *status, void *stream) {
  using namespace sb;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int s = check_topk_args(ld_emb, n_rows, dim, dim_pad, n_queries, k, capacity, out_ids, out_scores, status);
  if (s != SB_OK) return s;
  if (shadow_dtype != SB_DTYPE_F16 && shadow_dtype != SB_DTYPE_BF16) return SB_ERR_UNSUPPORTED;
  if (n_queries == 0) return SB_OK;
  if (queries == nullptr || out_ids == nullptr || stats == nullptr) return SB_ERR_INVALID_ARGUMENT;
  if (ld_q < dim || ld_16 < dim_pad) return SB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(emb16) % 16) || ((ld_16 * 2) % 16)) return SB_ERR_INVALID_ARGUMENT;
  const Workspace w = carve(workspace, n_queries, dim, dim_pad, capacity, n_rows);
  if (workspace == nullptr || workspace_bytes < w.bytes) return SB_ERR_WORKSPACE_TOO_SMALL;
  if (n_rows > 0) {
    if (emb == nullptr || emb16 == nullptr) return SB_ERR_INVALID_ARGUMENT;
    s = cosine_screen(emb16, ld_16, shadow_dtype, valid, n_rows, dim, dim_pad, stats, queries, ld_q, n_queries, k,
                      min_similarity, capacity, w, status, st);
    if (s != SB_OK) return s;
  }
  return cosine_rescore(emb, ld_emb, n_rows, dim, n_queries, k, min_similarity, id_offset, out_ids, out_scores,
                        capacity, w, status, st);
}

extern "C" SB_API int sb_topk_merge(const int64_t *ids, int64_t ids_list_stride, const float *scores,
                                    int64_t scores_list_stride, int32_t n_lists, int32_t n_queries, int32_t k,
                                    int64_t *out_ids, float *out_scores, void *stream) {
  if (n_lists < 1 || n_lists > 16 || n_queries < 0 || k < 1) return SB_ERR_INVALID_ARGUMENT;
  if (ids_list_stride < (int64_t)n_queries * k || scores_list_stride < (int64_t)n_queries * k)
    return SB_ERR_INVALID_ARGUMENT;
  if (n_queries == 0) return SB_OK;
  if (!ids || !scores || !out_ids || !out_scores) return SB_ERR_INVALID_ARGUMENT;
  if (k > 32) return SB_ERR_INVALID_ARGUMENT;
  const unsigned grid = (unsigned)((n_queries + sb::kMergeWarps - 1) / sb::kMergeWarps);
  const dim3 block(sb::kMergeWarps * 32);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (k <= 8)
    sb::topk_merge_kernel<8><<<grid, block, 0, st>>>(ids, ids_list_stride, scores, scores_list_stride, n_lists,
                                                     n_queries, k, out_ids, out_scores);
  else if (k <= 16)
    sb::topk_merge_kernel<16><<<grid, block, 0, st>>>(ids, ids_list_stride, scores, scores_list_stride, n_lists,
                                                      n_queries, k, out_ids, out_scores);
  else
    sb::topk_merge_kernel<32><<<grid, block, 0, st>>>(ids, ids_list_stride, scores, scores_list_stride, n_lists,
                                                      n_queries, k, out_ids, out_scores);
  return sb::launch_status();
}

// Partial-prefill attention over compacted query rows (sm_100a).
//
// For every compute row p of batch element b and query head h:
//     out[b, h, p] = softmax(q[b, h, p] . K[b, g(h), 0..p]^T * scale) V[b, g(h), 0..p]
// with g(h) = h / (Hq / Hkv) (grouped-query attention).  This is the
// reference's partial_prefill_attention (semblend_core/triton_kernels.py:
// 532-734), which runs one program per (row, head) with CUDA-core dot
// products, finds its row by scanning the mask and has no GQA.
//
// Tensor-core path (bf16 / fp16, head_dim 128): one CTA tile holds the
// G = Hq / Hkv query heads of a KV group at Pt = 128 / G consecutive compute
// rows (M = G * Pt <= 128 rows), so every K/V tile is read once for all heads
// sharing it and the rows of a tile share nearly the same causal bound.
//   warp 0     TMA producer: K and V tiles of 128 keys (3-stage ring)
//   warp 1     tcgen05.mma issuer: S = Q K^T into TMEM (double-buffered),
//              O += P V with P read from TMEM (kind::f16, fp32 accumulate)
//   warps 2-5  softmax: one row per thread; online softmax in the exp2
//              domain, P written back to TMEM over S, O rescaled in TMEM only
//              when the running max grows by more than 2^8 (exact: the final
//              normalisation uses the same reference max); then the epilogue.
// Work units (b, kv group, row tile) are assigned longest-first.
//
// CUDA-core path: any head_dim <= 256 and fp32 (the reference's own dtype in
// its tests), one CTA per (row, head), fp32 online softmax with expf.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <cmath>

#include "common.cuh"
#include "prof.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace sb {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 128;
// One pair of exponentials in every SB_ATTN_POLY_EVERY is evaluated as a
// polynomial on the FMA pipe instead of MUFU (0: all on MUFU).  All on MUFU
// measured fastest on B200 (c4 1,103 against 1,036-1,041 TFLOP/s for 1 in 4,
// 997 for 1 in 2; a c5 layer 978 against 923-929 and 877): the polynomial's
// 12 instructions a pair load the FMA pipe and the issue slots more than the
// MUFU time they save.
#ifndef SB_ATTN_POLY_EVERY
#define SB_ATTN_POLY_EVERY 0
#endif
constexpr int kPolyEvery = SB_ATTN_POLY_EVERY;

// warps 0-3 softmax of tile 0, warps 4-7 softmax of tile 1 (warpgroups 0 and 1),
// warp 8 TMA, warp 9 MMA, warps 10-11 idle (warpgroup 2).  Launched with 168
// registers a thread (384 x 168 fill the register file); warpgroup 2 gives
// registers up (setmaxnreg) so the softmax warpgroups can hold a whole S row:
// 2 x 128 x kSoftmaxRegs + 128 x kControlRegs = 384 x 168.
constexpr int kThreads = 384;
constexpr int kSoftmaxRegs = 200;
constexpr int kControlRegs = 104;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kControlRegs == kThreads * 168, "register split");
#ifndef SB_ATTN_K_STAGES
#define SB_ATTN_K_STAGES 2
#endif
constexpr int kKStages = SB_ATTN_K_STAGES;  // K ring (K is needed one MMA group before V)
constexpr int kVStages = 2;    // V ring
constexpr int kTileBytes = 128 * 128 * 2;  // one [128 x 128] 16-bit operand tile (two 64-column boxes)
constexpr int kHalfTile = kTileBytes / 2;
constexpr int kSmemBytes = 1024 + kTileBytes * (2 + kKStages + kVStages) + 256;
constexpr long long kWaitCycles = 2000000000LL;
// TMEM columns: tile t has S (P packed over its first half) at [256 t, 256 t + 128)
// and its O accumulator at [256 t + 128, 256 t + 256).
__host__ __device__ constexpr uint32_t tmem_s(int t) { return 256u * t; }
__host__ __device__ constexpr uint32_t tmem_o(int t) { return 256u * t + 128u; }

#if SB_ATTN_TRACE
__device__ long long g_trace[24 * 512];
#define SB_TRACE(slot, idx) do { if (blockIdx.x == 0 && (idx) < 512) g_trace[(slot) * 512 + (idx)] = clock64(); } while (0)
#else
#define SB_TRACE(slot, idx) do { } while (0)
#endif

struct AttnParams {
  const void *q;
  int64_t q_sb, q_sh, q_ss;
  void *out;
  int64_t o_sb, o_sh, o_ss;
  const int32_t *rows;
  int64_t rows_sb;
  const int32_t *counts;
  int B, Hq, Hkv, S, G, Pt, T_max;  // T_max: row-tile pairs of the longest batch element
  int64_t n_units;
  float scale_log2;
  int *status;
  unsigned *sched;  // [next unit, CTAs finished] of this launch's scheduler slot
};

// Work units are handed out dynamically (longest first): each CTA's producer
// thread takes the next unit index with an atomic add on a per-launch counter
// pair in device memory.  A launch takes one of kSchedSlots slots (round robin
// on the host); the last CTA to finish resets its slot, so up to kSchedSlots
// launches may be in flight on a device at once.
constexpr int kSchedSlots = 64;
__device__ unsigned g_attn_sched[kSchedSlots * 2];

// A work unit is two consecutive row tiles of one (batch element, KV group).
struct Unit {
  int b, g, r0;
  int n_rows[2];
  int nblk[2];
};

// Unit order: windows of kUnitWindow consecutive row-tile pairs, last window
// first (longest units first); inside a window every (batch, KV group) takes
// its kUnitWindow pairs in a row, so CTAs running at the same time share a few
// K/V streams in L2 instead of one per CTA.
#ifndef SB_ATTN_UNIT_WINDOW
#define SB_ATTN_UNIT_WINDOW 4
#endif
constexpr int kUnitWindow = SB_ATTN_UNIT_WINDOW;

__device__ __forceinline__ bool decode_unit(const AttnParams &P, int64_t u, Unit &w) {
  const int64_t bg_all = (int64_t)P.B * P.Hkv;
  const int64_t per_window = bg_all * kUnitWindow;
  const int64_t win = u / per_window, rem = u % per_window;
  const int bg = (int)(rem / kUnitWindow);
  const int tp = P.T_max - 1 - (int)(win * kUnitWindow + rem % kUnitWindow);
  if (tp < 0) return false;
  w.b = bg / P.Hkv;
  w.g = bg % P.Hkv;
  w.r0 = tp * 2 * P.Pt;
  const int cnt = P.counts[w.b];
  if (w.r0 >= cnt) return false;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int first = w.r0 + t * P.Pt;
    w.n_rows[t] = max(0, min(P.Pt, cnt - first));
    w.nblk[t] = w.n_rows[t] > 0 ? P.rows[(int64_t)w.b * P.rows_sb + first + w.n_rows[t] - 1] / kBN + 1 : 0;
  }
  return true;
}

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <> struct Pack2<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

// Two query tiles per CTA, processed in ping-pong: while the softmax warps of
// one tile turn its S block into P, the tensor cores run the other tile's
// P.V and next Q.K^T.  PV_t(j) is issued before S_t(j + 1), so the barrier
// that signals S_t(j + 1) also certifies that O_t holds blocks <= j.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const AttnParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sQ = smem;                          // [2] query tiles
  uint8_t *sK = sQ + 2 * kTileBytes;           // [kKStages]
  uint8_t *sV = sK + kKStages * kTileBytes;    // [kVStages]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sV + kVStages * kTileBytes);
  uint64_t *k_full = bars;                     // [kKStages <= 3]
  uint64_t *k_empty = bars + 3;                // [kKStages <= 3]
  uint64_t *v_full = bars + 6;                 // [kVStages]
  uint64_t *v_empty = bars + 8;                // [kVStages]
  uint64_t *q_full = bars + 10;                // [2]
  uint64_t *q_empty = bars + 12;
  uint64_t *s_full = bars + 13;                // [2]
  uint64_t *p_full = bars + 15;                // [2 tiles][2 key halves]
  uint64_t *o_final = bars + 19;               // [2]
  uint64_t *final_bar = bars + 21;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 22);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 23);
  uint64_t *unit_full = bars + 24;             // [2] unit ring: producer -> MMA + softmax warps
  uint64_t *unit_empty = bars + 26;            // [2]
  volatile int *unit_ring = reinterpret_cast<volatile int *>(bars + 28);  // [2]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kKStages; ++s) {
      tc::mbar_init(&k_full[s], 1);
      tc::mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      tc::mbar_init(&v_full[s], 1);
      tc::mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      tc::mbar_init(&q_full[t], 4);
      tc::mbar_init(&s_full[t], 1);
      tc::mbar_init(&p_full[2 * t], 4);
      tc::mbar_init(&p_full[2 * t + 1], 4);
      tc::mbar_init(&o_final[t], 1);
    }
    tc::mbar_init(q_empty, 1);
    tc::mbar_init(final_bar, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&unit_full[i], 1);
      tc::mbar_init(&unit_empty[i], 1 + 8);  // the MMA thread and the 8 softmax warps
    }
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 9) {
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
  pdl_wait();  // everything the previous kernel on this stream writes is visible from here on
  // n-th unit of this CTA (-1: no more work).  A whole warp (softmax) reads
  // the slot before lane 0 releases it; the single MMA thread releases it itself.
  auto pop_unit = [&](uint32_t n, bool whole_warp) -> int {
    if (!tc::mbar_wait(&unit_full[n & 1], (n >> 1) & 1, ab, 5, kWaitCycles)) return -1;
    const int u = unit_ring[n & 1];
    if (whole_warp) __syncwarp();
    if (!whole_warp || (threadIdx.x & 31) == 0) tc::mbar_arrive(&unit_empty[n & 1]);
    return u;
  };

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kControlRegs));
   if (warp == 8) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      tc::tma_prefetch_desc(&tmK);
      tc::tma_prefetch_desc(&tmV);
      uint32_t gl = 0, pushed = 0;
      bool ok = true, vfail = false;
      auto push_unit = [&](int u) -> bool {
        const uint32_t slot = pushed & 1, use = pushed >> 1;
        if (use > 0 && !tc::mbar_wait(&unit_empty[slot], (use - 1) & 1, ab, 2, kWaitCycles)) return false;
        unit_ring[slot] = u;
        tc::mbar_arrive(&unit_full[slot]);
        ++pushed;
        return true;
      };
      while (ok) {
        const int64_t u = atomicAdd(P.sched, 1u);
        if (u >= P.n_units) break;
        Unit w;
        if (!decode_unit(P, u, w)) continue;
        if (!push_unit((int)u)) {
          ok = false;
          break;
        }
        const int nb = max(w.nblk[0], w.nblk[1]);
        for (int j = 0; j < nb; ++j) {
          const uint32_t ks = gl % kKStages, kph = (gl / kKStages) & 1;
          const uint32_t vs = gl % kVStages, vph = (gl / kVStages) & 1;
          if (!tc::mbar_wait(&k_empty[ks], kph ^ 1, ab, 2, kWaitCycles)) {
            ok = false;
            break;
          }
          uint8_t *k_dst = sK + ks * kTileBytes;
          tc::mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
          tc::tma_load_4d(k_dst, &tmK, &k_full[ks], 0, j * kBN, w.g, w.b);
          tc::tma_load_4d(k_dst + kHalfTile, &tmK, &k_full[ks], 64, j * kBN, w.g, w.b);
          ++gl;  // the K load of this block is in flight from here on
          if (!tc::mbar_wait(&v_empty[vs], vph ^ 1, ab, 2, kWaitCycles)) {
            ok = false;
            vfail = true;
            break;
          }
          uint8_t *v_dst = sV + vs * kTileBytes;
          tc::mbar_arrive_expect_tx(&v_full[vs], kTileBytes);
          tc::tma_load_4d(v_dst, &tmV, &v_full[vs], 0, j * kBN, w.g, w.b);
          tc::tma_load_4d(v_dst + kHalfTile, &tmV, &v_full[vs], 64, j * kBN, w.g, w.b);
        }
      }
      if (ok) push_unit(-1);
      // every load this thread issued lands before the CTA can exit (the V load
      // of the last counted block is missing when its slot wait gave up)
      const uint32_t nk = gl < (uint32_t)kKStages ? gl : (uint32_t)kKStages;
      for (uint32_t i = gl - nk; i < gl; ++i)
        tc::mbar_wait(&k_full[i % kKStages], (i / kKStages) & 1, drain, 0, kWaitCycles);
      const uint32_t gv = vfail ? gl - 1 : gl;
      const uint32_t nv = gv < (uint32_t)kVStages ? gv : (uint32_t)kVStages;
      for (uint32_t i = gv - nv; i < gv; ++i)
        tc::mbar_wait(&v_full[i % kVStages], (i / kVStages) & 1, drain, 0, kWaitCycles);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ------------------------------
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_qk = tc::idesc_f16(kBM, kBN, fmt, 0);
      constexpr uint32_t idesc_pv = tc::idesc_f16(kBM, kD, fmt, 1);
      uint32_t gl = 0, qi = 0;
      uint32_t pc[2] = {0, 0};  // P blocks consumed per tile
      bool ok = true;
      // descriptors advance in 16-byte units of the start address (no carry out of its 14 bits)
      const uint64_t dq0 = tc::desc_kmajor_sw128(sQ);
      const uint64_t dk0 = tc::desc_kmajor_sw128(sK);
      const uint64_t dv0 = tc::desc_mnmajor_sw128(sV, 0, kHalfTile);
      constexpr uint32_t kTileUnits = kTileBytes >> 4, kHalfUnits = kHalfTile >> 4;
      auto issue_s = [&](int t, uint32_t st) {
        const uint32_t s_tmem = tmem + tmem_s(t);
        const uint64_t dq = dq0 + t * kTileUnits, dk = dk0 + st * kTileUnits;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16_ss(s_tmem, dq + kb * kHalfUnits + kk * 2, dk + kb * kHalfUnits + kk * 2, idesc_qk,
                            (kb | kk) != 0);
        tc::mma_commit(&s_full[t]);
      };
      for (uint32_t n = 0; ok; ++n) {
        const int u = pop_unit(n, false);
        if (u < 0) break;
        Unit w;
        decode_unit(P, u, w);
        const int nb = max(w.nblk[0], w.nblk[1]);
        if (!tc::mbar_wait(&q_full[0], qi & 1, ab, 3, kWaitCycles) ||
            !tc::mbar_wait(&q_full[1], qi & 1, ab, 3, kWaitCycles))
          break;
        tc::fence_after_sync();
        // S of block 0 for both tiles
        {
          const uint32_t ks = gl % kKStages;
          if (!tc::mbar_wait(&k_full[ks], (gl / kKStages) & 1, ab, 3, kWaitCycles)) break;
          tc::fence_after_sync();
          for (int t = 0; t < 2; ++t)
            if (w.nblk[t] > 0) issue_s(t, ks);
          tc::mma_commit(&k_empty[ks]);
        }
        for (int j = 0; j < nb && ok; ++j) {
          const uint32_t g = gl + j;
          const uint32_t vs = g % kVStages, vph = (g / kVStages) & 1;
          const uint32_t ks1 = (g + 1) % kKStages, kph1 = ((g + 1) / kKStages) & 1;
          bool v_ready = false, k_ready = false;
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= w.nblk[t]) continue;
            // P.V in two halves of 64 keys: the first runs while the softmax writes the second
            if (!tc::mbar_wait(&p_full[2 * t], pc[t] & 1, ab, 3, kWaitCycles)) {
              ok = false;
              break;
            }
            SB_TRACE(t, pc[t]);
            if (!v_ready) {
              if (!tc::mbar_wait(&v_full[vs], vph, ab, 3, kWaitCycles)) {
                ok = false;
                break;
              }
              v_ready = true;
            }
            SB_TRACE(20 + t, pc[t]);
            tc::fence_after_sync();
            const uint32_t p_tmem = tmem + tmem_s(t);
            const uint64_t dv = dv0 + vs * kTileUnits;
#pragma unroll
            for (int kk = 0; kk < kBN / 32; ++kk)
              tc::mma_bf16_ts(tmem + tmem_o(t), p_tmem + kk * 8, dv + kk * (2048 >> 4), idesc_pv,
                              (j == 0 && kk == 0) ? 0u : 1u);
            if (!tc::mbar_wait(&p_full[2 * t + 1], pc[t] & 1, ab, 3, kWaitCycles)) {
              ok = false;
              break;
            }
            SB_TRACE(16 + t, pc[t]);
            ++pc[t];
            tc::fence_after_sync();
#pragma unroll
            for (int kk = kBN / 32; kk < kBN / 16; ++kk)
              tc::mma_bf16_ts(tmem + tmem_o(t), p_tmem + kk * 8, dv + kk * (2048 >> 4), idesc_pv, 1u);
            if (j == w.nblk[t] - 1) tc::mma_commit(&o_final[t]);
            if (j + 1 < w.nblk[t]) {
              if (!k_ready) {
                if (!tc::mbar_wait(&k_full[ks1], kph1, ab, 3, kWaitCycles)) {
                  ok = false;
                  break;
                }
                tc::fence_after_sync();
                k_ready = true;
              }
              issue_s(t, ks1);
            }
            SB_TRACE(18 + t, pc[t] - 1);
          }
          if (!ok) break;
          tc::mma_commit(&v_empty[vs]);
          if (j + 1 < nb) tc::mma_commit(&k_empty[ks1]);
        }
        if (!ok) break;
        gl += nb;
        tc::mma_commit(q_empty);
        ++qi;
      }
      tc::mma_commit(final_bar);
      tc::mbar_wait(final_bar, 0, drain, 0, kWaitCycles);
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------ softmax / epilogue ------------------------------
    const int t = warp >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int m = quarter * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    uint32_t sc = 0, oc = 0, qi = 0;  // S blocks seen, O finals seen, units seen
    bool ok = true;
    const bool neg_scale = P.scale_log2 < 0.f;
    for (uint32_t n = 0; ok; ++n) {
      const int u = pop_unit(n, true);
      if (u < 0) break;
      Unit w;
      decode_unit(P, u, w);
      const int hh = m / P.Pt, pi = m - hh * P.Pt;
      const bool valid = hh < P.G && pi < w.n_rows[t];
      const int pos = valid ? P.rows[(int64_t)w.b * P.rows_sb + w.r0 + t * P.Pt + pi] : -1;
      const int head = w.g * P.G + hh;
      // gather this row of Q into the 128-byte-swizzled K-major tile (zeros for unused rows)
      if (t == 0 && quarter == 2 && lane == 0) SB_TRACE(22, qi);
      if (qi > 0 && !tc::mbar_wait(q_empty, (qi - 1) & 1, ab, 4, kWaitCycles)) break;
      {
        uint8_t *q_tile = sQ + t * kTileBytes;
        const uint4 *src = reinterpret_cast<const uint4 *>(
            reinterpret_cast<const T *>(P.q) + (valid ? (int64_t)w.b * P.q_sb + (int64_t)head * P.q_sh +
                                                            (int64_t)pos * P.q_ss
                                                      : 0));
        uint4 v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = valid ? src[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int kb = c >> 3, cc = c & 7;
          *reinterpret_cast<uint4 *>(q_tile + kb * kHalfTile + m * 128 + ((cc ^ (m & 7)) << 4)) = v[c];
        }
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&q_full[t]);
      ++qi;

      const int nb = w.nblk[t];
      float m_used = -INFINITY, l = 0.f;
      const uint32_t s_addr = tmem + lane_addr + tmem_s(t);
      for (int j = 0; j < nb; ++j) {
        if (!tc::mbar_wait(&s_full[t], sc & 1, ab, 4, kWaitCycles)) {
          ok = false;
          break;
        }
        if (quarter == 2 && lane == 0) SB_TRACE(2 + t, sc);
        ++sc;
        tc::fence_after_sync();
        const int key0 = j * kBN;
        // keys past this row are masked; unused rows (zero Q) are left unmasked and never stored
        const bool diag = valid && key0 + kBN - 1 > pos;
        const bool any_diag = __any_sync(0xffffffffu, diag);
        const float masked = neg_scale ? INFINITY : -INFINITY;
        // the whole S row of this thread, read from TMEM once
        uint32_t sr[kBN];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
        tc::tmem_ld_wait();
        if (any_diag) {
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (key0 + c > pos) sr[c] = __float_as_uint(masked);
        }
        float mx;
        {
          float a0 = masked, a1 = masked, a2 = masked, a3 = masked;
#pragma unroll
          for (int c = 0; c < kBN; c += 8) {
#define SB_X(i) __uint_as_float(sr[c + (i)])
            if (!neg_scale) {
              a0 = tc::max3(a0, SB_X(0), SB_X(1)), a1 = tc::max3(a1, SB_X(2), SB_X(3));
              a2 = tc::max3(a2, SB_X(4), SB_X(5)), a3 = tc::max3(a3, SB_X(6), SB_X(7));
            } else {
              a0 = tc::min3(a0, SB_X(0), SB_X(1)), a1 = tc::min3(a1, SB_X(2), SB_X(3));
              a2 = tc::min3(a2, SB_X(4), SB_X(5)), a3 = tc::min3(a3, SB_X(6), SB_X(7));
            }
#undef SB_X
          }
          mx = neg_scale ? fminf(fminf(a0, a1), fminf(a2, a3)) : fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
        }
        if (quarter == 2 && lane == 0) SB_TRACE(4 + t, sc);
        const float mx_s = mx * P.scale_log2;  // row max of the scaled logits (log2 domain)
        float m_new = m_used;
        bool need = false;
        if (mx_s > -INFINITY && (m_used == -INFINITY || mx_s > m_used + 8.f)) {
          need = m_used != -INFINITY;
          m_new = mx_s;
        }
        if (__any_sync(0xffffffffu, need)) {
          // O_t holds blocks < j (certified by this S block's barrier): rescale it in TMEM
          const float alpha = need ? tc::ex2_approx(m_used - m_new) : 1.f;
          const uint32_t o_addr = tmem + lane_addr + tmem_o(t);
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
            uint32_t r[32];
            tc::tmem_ld32(o_addr + c, r);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tc::tmem_st16(o_addr + c, *reinterpret_cast<const uint32_t(*)[16]>(r));
            tc::tmem_st16(o_addr + c + 16, *reinterpret_cast<const uint32_t(*)[16]>(r + 16));
          }
          tc::tmem_st_wait();
          l *= alpha;
        }
        m_used = m_new;
        // P = 2^(s * scale_log2 - m_used): masked keys (+-inf) and rows with no
        // visible key yet (m_used = -inf) give 0
        const float neg_m = m_used != -INFINITY ? -m_used : -INFINITY;
        const float2 cc = make_float2(P.scale_log2, P.scale_log2), nm = make_float2(neg_m, neg_m);
        float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < kBN; c += 32) {
          uint32_t r[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 e = tc::fma2(make_float2(__uint_as_float(sr[c + 2 * i]), __uint_as_float(sr[c + 2 * i + 1])),
                                      cc, nm);
            const float2 pp = (kPolyEvery > 0 && i % (kPolyEvery > 0 ? kPolyEvery : 1) == kPolyEvery - 1)
                                  ? tc::exp2_poly2(e)
                                  : make_float2(tc::ex2_approx(e.x), tc::ex2_approx(e.y));
            sum2 = tc::add2(sum2, pp);
            r[i] = Pack2<T>::pack(pp.x, pp.y);
          }
          tc::tmem_st16(s_addr + c / 2, r);
          if (c % 64 == 32) {  // a half of P (64 keys) is in TMEM: let its P.V start
            tc::tmem_st_wait();
            tc::fence_before_sync();
            __syncwarp();
            if (c == kBN - 32) {
              if (quarter == 2 && lane == 0) SB_TRACE(6 + t, sc);
              if (lane == 0) SB_TRACE(8 + 4 * t + quarter, sc);
            }
            if (lane == 0) tc::mbar_arrive(&p_full[2 * t + c / 64]);
          }
        }
        l += sum2.x + sum2.y;
      }
      if (!ok) break;
      if (nb == 0) continue;
      // epilogue: O / l for this row
      if (!tc::mbar_wait(&o_final[t], oc & 1, ab, 4, kWaitCycles)) break;
      ++oc;
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4 *dst = reinterpret_cast<uint4 *>(
          reinterpret_cast<T *>(P.out) +
          (valid ? (int64_t)w.b * P.o_sb + (int64_t)head * P.o_sh + (int64_t)pos * P.o_ss : 0));
      const uint32_t o_addr = tmem + lane_addr + tmem_o(t);
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        uint32_t r[32];
        tc::tmem_ld32(o_addr + c, r);
        tc::tmem_ld_wait();
        if (valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = Pack2<T>::pack(__uint_as_float(r[2 * i]) * inv, __uint_as_float(r[2 * i + 1]) * inv);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[c / 8 + i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      if (t == 0 && quarter == 2 && lane == 0) SB_TRACE(23, qi - 1);
      tc::fence_before_sync();
    }
  }

  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 9) tc::tmem_dealloc(tmem, 512);
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

// ---------------------------------------------------------------------------
// CUDA-core path
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(const T *__restrict__ q, const T *__restrict__ k,
                                                        const T *__restrict__ v, T *__restrict__ out, AttnParams P,
                                                        int64_t k_sb, int64_t k_sh, int64_t k_ss, int64_t v_sb,
                                                        int64_t v_sh, int64_t v_ss, int D, float scale) {
  const int r = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  if (r >= P.counts[b]) return;
  const int pos = P.rows[(int64_t)b * P.rows_sb + r];
  const int g = h / P.G;
  __shared__ float qs[256];
  __shared__ float ps[128];
  __shared__ float red[4];
  const int tid = threadIdx.x;
  for (int d = tid; d < D; d += 128)
    qs[d] = Elem<T>::to_f32(q[(int64_t)b * P.q_sb + (int64_t)h * P.q_sh + (int64_t)pos * P.q_ss + d]);
  __syncthreads();
  const T *kb = k + (int64_t)b * k_sb + (int64_t)g * k_sh;
  const T *vb = v + (int64_t)b * v_sb + (int64_t)g * v_sh;
  float mrun = -INFINITY, lrun = 0.f, acc0 = 0.f, acc1 = 0.f;
  for (int k0 = 0; k0 <= pos; k0 += 128) {
    const int key = k0 + tid;
    float sc = -INFINITY;
    if (key <= pos) {
      float dot = 0.f;
      const T *kr = kb + (int64_t)key * k_ss;
      for (int d = 0; d < D; ++d) dot = fmaf(qs[d], Elem<T>::to_f32(kr[d]), dot);
      sc = dot * scale;
    }
    float mx = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    const float m_new = fmaxf(mrun, mx);
    const float corr = mrun == -INFINITY ? 0.f : expf(mrun - m_new);
    const float p = key <= pos ? expf(sc - m_new) : 0.f;
    ps[tid] = p;
    float sum = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    sum = red[0] + red[1] + red[2] + red[3];
    lrun = lrun * corr + sum;
    const int nk = min(128, pos + 1 - k0);
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < nk; ++j) {
      const T *vr = vb + (int64_t)(k0 + j) * v_ss;
      const float pj = ps[j];
      if (tid < D) a0 = fmaf(pj, Elem<T>::to_f32(vr[tid]), a0);
      if (tid + 128 < D) a1 = fmaf(pj, Elem<T>::to_f32(vr[tid + 128]), a1);
    }
    acc0 = acc0 * corr + a0;
    acc1 = acc1 * corr + a1;
    mrun = m_new;
    __syncthreads();
  }
  T *o = out + (int64_t)b * P.o_sb + (int64_t)h * P.o_sh + (int64_t)pos * P.o_ss;
  if (tid < D) o[tid] = Elem<T>::from_f32(acc0 / lrun);
  if (tid + 128 < D) o[tid + 128] = Elem<T>::from_f32(acc1 / lrun);
}

// Compute-mask -> sorted row indices and counts, one CTA per batch element.
__global__ void mask_to_rows_kernel(const uint8_t *__restrict__ mask, int64_t mask_sb, int S,
                                    int32_t *__restrict__ rows, int64_t rows_sb, int32_t *__restrict__ counts) {
  const int b = blockIdx.x;
  __shared__ int warp_tot[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int s0 = 0; s0 < S; s0 += blockDim.x) {
    const int s = s0 + threadIdx.x;
    const int f = (s < S && mask[(int64_t)b * mask_sb + s]) ? 1 : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    const int before = __popc(bal & ((1u << lane) - 1));
    if (lane == 0) warp_tot[wid] = __popc(bal);
    __syncthreads();
    int off = 0, tot = 0;
    for (int i = 0; i < nw; ++i) {
      if (i < wid) off += warp_tot[i];
      tot += warp_tot[i];
    }
    if (f) rows[(int64_t)b * rows_sb + base + off + before] = s;
    __syncthreads();
    if (threadIdx.x == 0) base += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[b] = base;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

// This launch's scheduler counter pair on the current device (the symbol's
// address is looked up once per device, with that device current).
unsigned *sched_slot() {
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
      e = cudaGetSymbolAddress(&p, g_attn_sched);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return nullptr;
      }
      base[dev] = static_cast<unsigned *>(p);
    }
  }
  return base[dev] + 2 * (next.fetch_add(1) % kSchedSlots);
}

template <typename T>
int launch_tc(const sb_attn_tensor &k, const sb_attn_tensor &v, const AttnParams &P, CUtensorMapDataType dt,
              cudaStream_t st) {
  CUtensorMap tk, tv;
  const uint64_t es = sizeof(T);
  if (!make_tmap_4d(&tk, dt, k.data, kD, P.S, P.Hkv, P.B, k.stride_seq * es, k.stride_head * es,
                    k.stride_batch * es, 64, kBN) ||
      !make_tmap_4d(&tv, dt, v.data, kD, P.S, P.Hkv, P.B, v.stride_seq * es, v.stride_head * es,
                    v.stride_batch * es, 64, kBN))
    return SB_ERR_CUDA;
  if (ensure_dynamic_smem(reinterpret_cast<const void *>(attn_tc_kernel<T>), kSmemBytes) != SB_OK) return SB_ERR_CUDA;
  AttnParams Pl = P;
  Pl.sched = sched_slot();
  if (Pl.sched == nullptr) return SB_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(sm_count(), P.n_units);
  const int slot = prof_before(st);
  const cudaError_t e = launch_pdl(attn_tc_kernel<T>, dim3(grid), dim3(kThreads), kSmemBytes, st, tk, tv, Pl);
  prof_after(slot, st);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  return launch_status();
}

template <typename T>
int launch_simt(const sb_attn_tensor &q, const sb_attn_tensor &k, const sb_attn_tensor &v,
                const sb_attn_tensor &out, const AttnParams &P, int D, float scale, int max_rows, cudaStream_t st) {
  dim3 grid((unsigned)max_rows, (unsigned)P.Hq, (unsigned)P.B);
  const int slot = prof_before(st);
  attn_simt_kernel<T><<<grid, 128, 0, st>>>(
      reinterpret_cast<const T *>(q.data), reinterpret_cast<const T *>(k.data), reinterpret_cast<const T *>(v.data),
      reinterpret_cast<T *>(out.data), P, k.stride_batch, k.stride_head, k.stride_seq, v.stride_batch,
      v.stride_head, v.stride_seq, D, scale);
  prof_after(slot, st);
  return launch_status();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace sb

#if SB_ATTN_TRACE
extern "C" SB_API int sb_attn_trace_read(long long *dst) {
  return cudaMemcpyFromSymbol(dst, sb::g_trace, sizeof(long long) * 24 * 512) == cudaSuccess ? 0 : -3;
}
#endif

extern "C" SB_API int sb_mask_to_rows(const uint8_t *mask, int64_t mask_stride, int32_t batch, int32_t seq_len,
                                      int32_t *rows, int64_t rows_stride, int32_t *counts, void *stream) {
  if (batch < 0 || seq_len < 0) return SB_ERR_INVALID_ARGUMENT;
  if (batch == 0) return SB_OK;
  if (!mask || !rows || !counts || rows_stride < seq_len) return SB_ERR_INVALID_ARGUMENT;
  sb::mask_to_rows_kernel<<<batch, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(mask, mask_stride, seq_len,
                                                                                       rows, rows_stride, counts);
  return sb::launch_status();
}

extern "C" SB_API int sb_partial_attention(sb_attn_tensor q, sb_attn_tensor k, sb_attn_tensor v, sb_attn_tensor out,
                                           const int32_t *rows, int64_t rows_stride, const int32_t *counts,
                                           int32_t max_rows, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                           int32_t seq_len, int32_t head_dim, float scale, int32_t dtype,
                                           int32_t *status, void *stream) {
  using namespace sb;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (batch < 0 || n_q_heads <= 0 || n_kv_heads <= 0 || seq_len < 0 || head_dim <= 0 || max_rows < 0)
    return SB_ERR_INVALID_ARGUMENT;
  if (n_q_heads % n_kv_heads) return SB_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0 || max_rows == 0) return SB_OK;
  if (!q.data || !k.data || !v.data || !out.data || !rows || !counts || !status) return SB_ERR_INVALID_ARGUMENT;
  if (head_dim > 256) return SB_ERR_UNSUPPORTED;
  if (elem_bytes(dtype) == 0) return SB_ERR_UNSUPPORTED;
  AttnParams P;
  P.q = q.data;
  P.q_sb = q.stride_batch, P.q_sh = q.stride_head, P.q_ss = q.stride_seq;
  P.out = out.data;
  P.o_sb = out.stride_batch, P.o_sh = out.stride_head, P.o_ss = out.stride_seq;
  P.rows = rows;
  P.rows_sb = rows_stride;
  P.counts = counts;
  P.B = batch, P.Hq = n_q_heads, P.Hkv = n_kv_heads, P.S = seq_len;
  P.G = n_q_heads / n_kv_heads;
  P.status = status;
  const int es = elem_bytes(dtype);
  const bool tc_ok = dtype != SB_DTYPE_F32 && head_dim == kD && P.G <= kBM && std::isfinite(scale) && scale != 0.f &&
                     aligned16(q.data) &&
                     aligned16(out.data) && aligned16(k.data) && aligned16(v.data) && (q.stride_seq * es) % 16 == 0 &&
                     (q.stride_head * es) % 16 == 0 && (q.stride_batch * es) % 16 == 0 &&
                     (out.stride_seq * es) % 16 == 0 && (out.stride_head * es) % 16 == 0 &&
                     (out.stride_batch * es) % 16 == 0 && (k.stride_seq * es) % 16 == 0 &&
                     (k.stride_head * es) % 16 == 0 && (k.stride_batch * es) % 16 == 0 &&
                     (v.stride_seq * es) % 16 == 0 && (v.stride_head * es) % 16 == 0 &&
                     (v.stride_batch * es) % 16 == 0;
  if (tc_ok) {
    P.Pt = kBM / P.G;
    P.T_max = (max_rows + 2 * P.Pt - 1) / (2 * P.Pt);
    P.n_units = (int64_t)((P.T_max + kUnitWindow - 1) / kUnitWindow) * kUnitWindow * batch * n_kv_heads;
    P.scale_log2 = scale * 1.4426950408889634f;
    if (dtype == SB_DTYPE_BF16) return launch_tc<__nv_bfloat16>(k, v, P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
    return launch_tc<__half>(k, v, P, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
  }
  P.Pt = 1;
  if (max_rows > 0x7fffffff) return SB_ERR_TOO_LARGE;
  if (n_q_heads > 65535 || batch > 65535) return SB_ERR_TOO_LARGE;
  switch (dtype) {
    case SB_DTYPE_F32: return launch_simt<float>(q, k, v, out, P, head_dim, scale, max_rows, st);
    case SB_DTYPE_F16: return launch_simt<__half>(q, k, v, out, P, head_dim, scale, max_rows, st);
    default: return launch_simt<__nv_bfloat16>(q, k, v, out, P, head_dim, scale, max_rows, st);
  }
}

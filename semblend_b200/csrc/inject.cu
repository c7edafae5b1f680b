// Fused donor-KV gather + RoPE correction + paged / flat scatter (sm_100a).
//
// One launch covers every descriptor (request) of a call and every
// (layer, kv, head) row of each pair.  A CTA owns a tile of pairs and a chunk
// of (layer, kv, head) units: its threads compute cos/sin of their pair's
// angles once and reuse them for every K row of the chunk, so the
// transcendental cost is amortised over layers and heads and the kernel stays
// bound by HBM traffic.  Each thread moves two vectors of up to 16 bytes per
// row (the two halves of its RoPE pairs), with streaming loads and stores.
//
// Arithmetic follows the reference's CPU path term by term
// (semblend_core/rope_correction.py:304-328 for delta correction,
// :806-823 for the NoPE two-step, :753-779 for a constant delta):
// theta = fp32(position difference) * inv_freq[i] as one fp32 multiply, and
// every product and sum of the rotation rounded separately (no FMA
// contraction), so results differ from the reference only where the cos/sin
// values themselves differ in their last bit.  Out-of-range pairs are skipped
// the way the reference's Triton kernels skip them
// (rope_correction.py:117-129, triton_kernels.py:106-108, :246-260) and are
// counted in a device error counter.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include <cuda.h>

#include "common.cuh"
#include "prof.cuh"
#include "tcgen05.cuh"

namespace sb {
namespace {

#ifndef SB_INJECT_MIN_BLOCKS
#define SB_INJECT_MIN_BLOCKS 4  // resident CTAs per SM the register budget targets
#endif
#ifndef SB_INJECT_TARGET_WAVES
#define SB_INJECT_TARGET_WAVES 16  // waves of resident CTAs a large launch aims for
#endif
#ifndef SB_INJECT_MIN_ROWS
#define SB_INJECT_MIN_ROWS 18  // rows per thread at least, in a launch of many pair tiles (swept: 8-18)
#endif
#ifndef SB_INJECT_UNROLL
#define SB_INJECT_UNROLL 2  // rows in flight per thread
#endif
constexpr int kThreads = 256;
constexpr int kUnroll = SB_INJECT_UNROLL;

struct InjectCommon {
  sb_inject_params p;
  unsigned long long *err;
  int32_t n_desc;
  int32_t pairs_per_tile;
  int32_t tpr;  // threads per row
  int32_t n_kv_sel;
  int32_t kv_first;
  int32_t units_per_chunk;
  int64_t n_units;
};

// Descriptors in the kernel parameters (up to MAXD of them)...
template <int MAXD> struct InjectLaunch {
  InjectCommon c;
  int64_t tile_start[MAXD + 1];
  sb_inject_desc desc[MAXD];
};

// ... or in a device table (any number): tile_start[n_desc + 1] after desc[n_desc].
struct InjectLaunchTable {
  InjectCommon c;
  const sb_inject_desc *desc;
  const int64_t *tile_start;
};

// The descriptor owning pair tile `tile` and that descriptor's first tile.
template <int MAXD>
__device__ __forceinline__ const sb_inject_desc &find_desc(const InjectLaunch<MAXD> &L, int64_t tile,
                                                           int64_t &first) {
  int di = 0;
#pragma unroll 1
  while (di + 1 < L.c.n_desc && tile >= L.tile_start[di + 1]) ++di;
  first = L.tile_start[di];
  return L.desc[di];
}

__device__ __forceinline__ const sb_inject_desc &find_desc(const InjectLaunchTable &L, int64_t tile,
                                                           int64_t &first) {
  // the last descriptor whose first tile is <= tile (descriptors without pairs own no tile)
  int lo = 0, hi = L.c.n_desc - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(L.tile_start + mid) <= tile) lo = mid; else hi = mid - 1;
  }
  first = __ldg(L.tile_start + lo);
  return L.desc[lo];
}

__device__ __forceinline__ bool resolve_row(const sb_rows &r, int64_t pos, int64_t &off) {
  if (pos < 0) return false;
  if (r.block_table == nullptr) {
    if (pos >= r.n_logical) return false;
    off = pos * r.stride_pos;
    return true;
  }
  const int64_t lb = pos / r.block_size;
  if (lb >= r.n_logical) return false;
  const int64_t phys = load_index(r.block_table, lb, r.block_table_dtype);
  if (phys < 0 || phys >= r.n_physical) return false;
  off = phys * r.stride_block + (pos - lb * r.block_size) * r.stride_pos;
  return true;
}

template <typename T>
__device__ __forceinline__ T *layer_base(const sb_rows &r, int l) {
  if (r.layer_ptrs != nullptr) return reinterpret_cast<T *>(r.layer_ptrs[l]);
  return reinterpret_cast<T *>(r.base) + (int64_t)l * r.stride_layer;
}

// cos / sin of an fp32 angle: evaluated in double precision and rounded once,
// which gives the correctly rounded fp32 value in all but rare cases.
__device__ __forceinline__ void sincos_f32(float theta, float &s, float &c) {
  double sd, cd;
  sincos((double)theta, &sd, &cd);
  s = (float)sd;
  c = (float)cd;
}

// (x, y) <- (x*c - y*s, x*s + y*c); every product and sum rounded on its own.
__device__ __forceinline__ void rotate_fwd(float &x, float &y, float c, float s) {
  const float nx = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
  const float ny = __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c));
  x = nx;
  y = ny;
}
// (x, y) <- (x*c + y*s, (-x)*s + y*c): rotation by the negated angle.
__device__ __forceinline__ void rotate_inv(float &x, float &y, float c, float s) {
  const float nx = __fadd_rn(__fmul_rn(x, c), __fmul_rn(y, s));
  const float ny = __fadd_rn(__fmul_rn(-x, s), __fmul_rn(y, c));
  x = nx;
  y = ny;
}

template <typename T, bool NOPE>
__device__ __forceinline__ void rotate_pair(T &a, T &b, float c1, float s1, float c2, float s2) {
  float x = Elem<T>::to_f32(a), y = Elem<T>::to_f32(b);
  if (NOPE) {
    rotate_inv(x, y, c1, s1);
    rotate_fwd(x, y, c2, s2);
  } else {
    rotate_fwd(x, y, c1, s1);
  }
  a = Elem<T>::from_f32(x);
  b = Elem<T>::from_f32(y);
}

// c2 / s2 hold the second angle of the NoPE two-step and have one (unused)
// slot otherwise.
template <typename T, int VEC, bool NOPE>
__device__ __forceinline__ void rotate_vectors(Vec<T, VEC> &va, Vec<T, VEC> &vb, bool neox,
                                               const float *c1, const float *s1,
                                               const float *c2, const float *s2) {
  constexpr int kSlots2 = NOPE ? VEC : 1;
  if (neox || VEC == 1) {
    // element e of va pairs with element e of vb (frequency slot e)
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      rotate_pair<T, NOPE>(va.e[e], vb.e[e], c1[e], s1[e], c2[e % kSlots2], s2[e % kSlots2]);
  } else {
    // interleaved: adjacent elements pair up; va holds slots [0, VEC/2),
    // vb holds slots [VEC/2, VEC)
#pragma unroll
    for (int m = 0; m < VEC / 2; ++m) {
      const int a = m, b = VEC / 2 + m;
      rotate_pair<T, NOPE>(va.e[2 * m], va.e[2 * m + 1], c1[a], s1[a], c2[a % kSlots2], s2[a % kSlots2]);
      rotate_pair<T, NOPE>(vb.e[2 * m], vb.e[2 * m + 1], c1[b], s1[b], c2[b % kSlots2], s2[b % kSlots2]);
    }
  }
}

// The angles of each pair (the RoPE rotation's theta = m * inv_freq[f] for the
// pair's position difference, constant or NoPE positions m).
__device__ __forceinline__ void pair_angles(const sb_inject_params &P, int64_t sp, int64_t tp, float &m1,
                                           float &m2) {
  m2 = 0.f;
  if (P.k_angle == SB_ANGLE_DELTA) {
    m1 = (float)(tp - sp);
  } else if (P.k_angle == SB_ANGLE_CONST) {
    m1 = (float)P.const_delta;
  } else {
    m1 = (float)sp;
    m2 = (float)tp;
  }
}

// cos / sin of this thread's VEC frequency slots for its pair's angle(s),
// computed once per tile for every run of consecutive pairs with the same
// angles and read from a shared table: chunk-shifted donors give a 32-pair tile
// one or two runs, so a CTA evaluates a few hundred double-precision sincos
// instead of one set per thread (2,048 for a 256-thread CTA at VEC 8).
// The kThreads threads that own the pair slots all call it: it synchronises
// them with the block barrier, or with named barrier 1 when NAMED (the
// bulk-staged kernel's consumers, whose producer warp runs on its own).
// Threads whose pair is not valid get nothing written.
template <bool NAMED>
__device__ __forceinline__ void pair_slots_sync() {
  if (NAMED)
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
  else
    __syncthreads();
}

template <int VEC, bool NOPE, bool NAMED>
__device__ __forceinline__ void tile_angles(const sb_inject_params &P, int ppt, int pl, int slice, bool ok,
                                            float m1, float m2, float *c1, float *s1, float *c2, float *s2) {
  constexpr int kA = NOPE ? 2 : 1;
  __shared__ float key[kA][kThreads];
  __shared__ uint8_t valid[kThreads];
  __shared__ int16_t run_of[kThreads];
  __shared__ float run_key[kA][kThreads];
  __shared__ int warp_starts[kThreads / 32];
  __shared__ float2 table[kA][kThreads * VEC];  // (cos, sin) per (run, frequency slot)
  const int t = threadIdx.x;
  if (slice == 0 && pl < ppt && t < kThreads) {
    key[0][pl] = m1;
    if (NOPE) key[kA - 1][pl] = m2;
    valid[pl] = ok ? 1 : 0;
  }
  pair_slots_sync<NAMED>();
  // run starts among the tile's valid pair slots, numbered by a block-wide count
  bool start = false;
  if (t < ppt && valid[t]) {
    start = t == 0 || !valid[t - 1] || key[0][t] != key[0][t - 1] || (NOPE && key[kA - 1][t] != key[kA - 1][t - 1]);
  }
  const unsigned bal = __ballot_sync(0xffffffffu, start);
  const int lane = t & 31, w = t >> 5;
  if (lane == 0 && w < kThreads / 32) warp_starts[w] = __popc(bal);
  pair_slots_sync<NAMED>();
  int before = 0, n_runs = 0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) {
    before += i < w ? warp_starts[i] : 0;
    n_runs += warp_starts[i];
  }
  const int upto = before + __popc(bal & (lane == 31 ? 0xffffffffu : ((2u << lane) - 1u)));
  if (t < ppt) run_of[t] = (int16_t)(upto - 1);  // -1: an invalid slot before any valid one
  if (start) {
    run_key[0][upto - 1] = key[0][t];
    if (NOPE) run_key[kA - 1][upto - 1] = key[kA - 1][t];
  }
  pair_slots_sync<NAMED>();
  const int half = P.head_dim / 2;
  for (int e = t; e < n_runs * half; e += kThreads) {
    const int r = e / half, f = e - r * half;
    const float inv = P.inv_freq[f];
    float sv, cv;
    sincos_f32(__fmul_rn(run_key[0][r], inv), sv, cv);
    table[0][e] = make_float2(cv, sv);
    if (NOPE) {
      sincos_f32(__fmul_rn(run_key[kA - 1][r], inv), sv, cv);
      table[kA - 1][e] = make_float2(cv, sv);
    }
  }
  pair_slots_sync<NAMED>();
  if (ok) {
    const int base = run_of[pl] * half + slice * VEC;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float2 a = table[0][base + e];
      c1[e] = a.x;
      s1[e] = a.y;
      if (NOPE) {
        const float2 b = table[kA - 1][base + e];
        c2[e % (NOPE ? VEC : 1)] = b.x;
        s2[e % (NOPE ? VEC : 1)] = b.y;
      }
    }
  }
}

template <typename T, int VEC, typename LT, bool NOPE>
__global__ void __launch_bounds__(kThreads, SB_INJECT_MIN_BLOCKS)
    inject_kernel(const __grid_constant__ LT L) {
  const InjectCommon &C = L.c;
  const int tpr = C.tpr;
  const int pl = threadIdx.x / tpr;
  const int slice = threadIdx.x - pl * tpr;
  const int64_t tile = blockIdx.x;
  int64_t first;
  // A descriptor in the kernel parameters is read from the constant bank.  One
  // in a device table sits in global memory, which the row loop's stores could
  // alias as far as the compiler knows, so it would be read again for every
  // row: the CTA's descriptor (all its pairs share one) is copied to shared
  // memory first.
  __shared__ sb_inject_desc s_desc;
  __shared__ int64_t s_first;
  const sb_inject_desc *dp;
  if constexpr (std::is_same<LT, InjectLaunchTable>::value) {
    if (threadIdx.x == 0) {
      s_desc = find_desc(L, tile, s_first);
    }
    __syncthreads();
    dp = &s_desc;
    first = s_first;
  } else {
    dp = &find_desc(L, tile, first);
  }
  const sb_inject_desc &d = *dp;
  const sb_inject_params &P = C.p;
  // no thread leaves before the angle table's barriers: threads past the tile's
  // pairs, or past the descriptor's last pair, take part with no pair
  const int64_t pair = (tile - first) * C.pairs_per_tile + pl;
  const bool has_pair = pl < C.pairs_per_tile && pair < d.n_pairs;
  int64_t sp = 0, tp = 0, soff = 0, doff = 0, chk = 0;
  bool ok = false;
  if (has_pair) {
    sp = load_index(d.src_pos, pair, d.pos_dtype);
    tp = load_index(d.dst_pos, pair, d.pos_dtype);
    const int64_t srow =
        d.src_row == SB_ROW_AT_PAIR ? pair : (d.src_row == SB_ROW_AT_DST_POS ? tp : sp);
    const int64_t drow =
        d.dst_row == SB_ROW_AT_PAIR ? pair : (d.dst_row == SB_ROW_AT_SRC_POS ? sp : tp);
    ok = resolve_row(d.src, srow, soff) && resolve_row(d.dst, drow, doff);
    if (ok && (d.flags & SB_DESC_CHECK_SRC_IN_DST)) ok = resolve_row(d.dst, sp, chk);
    if (!ok && blockIdx.y == 0 && slice == 0 && C.err != nullptr) atomicAdd(C.err, 1ull);
  }

  const int D = P.head_dim;
  const bool neox = P.rotary_style == SB_ROTARY_NEOX;
  int oa, ob;
  if (neox) {
    oa = slice * VEC;
    ob = D / 2 + slice * VEC;
  } else if (VEC == 1) {
    oa = 2 * slice;
    ob = 2 * slice + 1;
  } else {
    oa = 2 * slice * VEC;
    ob = oa + VEC;
  }

  const bool rot = P.k_angle != SB_ANGLE_NONE && (P.kv_select & SB_KV_K);
  // c2 / s2 (the second angle) only exist in the NoPE instantiation
  float c1[VEC], s1[VEC], c2[NOPE ? VEC : 1], s2[NOPE ? VEC : 1];
#pragma unroll
  for (int e = 0; e < VEC; ++e) c1[e] = 1.f, s1[e] = 0.f;
#pragma unroll
  for (int e = 0; e < (NOPE ? VEC : 1); ++e) c2[e] = 1.f, s2[e] = 0.f;
  if (rot) {  // uniform over the block
    float m1 = 0.f, m2 = 0.f;
    if (ok) pair_angles(P, sp, tp, m1, m2);
    tile_angles<VEC, NOPE, false>(P, C.pairs_per_tile, pl, slice, ok, m1, m2, c1, s1, c2, s2);
  }
  if (!ok) return;

  const int H = P.n_heads;
  // units are numbered (layer, kv, head) with the head fastest; n_units < 2^31
  const int ua = (int)((int64_t)blockIdx.y * C.units_per_chunk);
  const int nrow = (int)min((int64_t)C.units_per_chunk, C.n_units - ua);
  const int64_t sdim = d.src.stride_dim, ddim = d.dst.stride_dim;
  // (layer, kv, head) cursor of the next row, advanced one unit per row
  int h = ua % H, kvi = (ua / H) % C.n_kv_sel, l = (ua / H) / C.n_kv_sel;

#pragma unroll 1
  for (int i0 = 0; i0 < nrow; i0 += kUnroll) {
    Vec<T, VEC> va[kUnroll], vb[kUnroll];
    T *dptr[kUnroll];
    bool krow[kUnroll];
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      dptr[r] = nullptr;
      krow[r] = false;
      if (i0 + r < nrow) {
        const int kv = C.kv_first + kvi;
        const T *s = layer_base<T>(d.src, l) + kv * d.src.stride_kv + h * d.src.stride_head + soff;
        T *t = layer_base<T>(d.dst, l) + kv * d.dst.stride_kv + h * d.dst.stride_head + doff;
        if (++h == H) {
          h = 0;
          if (++kvi == C.n_kv_sel) {
            kvi = 0;
            ++l;
          }
        }
        if (VEC == 1) {
          va[r].e[0] = s[oa * sdim];
          vb[r].e[0] = s[ob * sdim];
        } else {
          load_vec(va[r], s + oa);
          load_vec(vb[r], s + ob);
        }
        dptr[r] = t;
        krow[r] = kv == 0;
      }
    }
#pragma unroll
    for (int r = 0; r < kUnroll; ++r) {
      if (dptr[r] == nullptr) continue;
      if (rot && krow[r]) rotate_vectors<T, VEC, NOPE>(va[r], vb[r], neox, c1, s1, c2, s2);
      if (VEC == 1) {
        dptr[r][oa * ddim] = va[r].e[0];
        dptr[r][ob * ddim] = vb[r].e[0];
      } else {
        store_vec(dptr[r] + oa, va[r]);
        store_vec(dptr[r] + ob, vb[r]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy-staged variant.  The same work split as inject_kernel (a CTA owns a
// tile of pairs and a chunk of (layer, kv, head) units, a consumer thread owns
// one pair and the two 16-byte halves of its RoPE pairs), but the source rows
// reach shared memory through 1-D cp.async.bulk copies issued by one producer
// thread: for every unit, the tile's source rows (one copy per run of
// contiguous rows: chunk-shifted donors give runs of up to the whole tile) land
// in a ring of kBulkStages stages of 8 KB, so each CTA keeps up to
// kBulkStages x 8 KB of reads in flight without holding them in registers.
// Consumers rotate K in registers and store 16-byte vectors to the destination
// rows.  Selected by SB_INJECT_BULK_STAGED when every row is a whole number of
// 16-byte vectors at 16-byte aligned addresses (the copies' alignment rule).
// Measured against the direct path on B200: slower on c2 (1.93-1.96 against
// 1.77 ms: a 32-pair tile there breaks into ~5 runs at the recompute holes,
// and the donor chunks that overlap are served by L2 either way) and on c1,
// within 3 % faster on c5 (whole 256-token chunks: one copy a unit).  Every wait is bounded: a
// stalled pipeline (never expected: producer and consumers are the same CTA)
// gives up, counts the tile's pairs as skipped, and the producer waits for the
// copies it has in flight before the CTA exits.
// ---------------------------------------------------------------------------
#ifndef SB_INJECT_BULK_STAGES
#define SB_INJECT_BULK_STAGES 3
#endif
constexpr int kBulkStages = SB_INJECT_BULK_STAGES;
constexpr int kBulkConsumers = kThreads;             // 8 warps, as inject_kernel
constexpr int kBulkThreads = kBulkConsumers + 32;    // + the producer warp
constexpr int kStageBytes = kBulkConsumers * 32;     // pairs of a tile x row bytes (2 x 16 B per thread)
constexpr long long kBulkWaitCycles = 1LL << 31;     // about a second
constexpr size_t kBulkDynSmem = (size_t)kBulkStages * kStageBytes + 128;

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(tc::smem_u32(bar))
      : "memory");
}

template <typename T, typename LT, bool NOPE>
__global__ void __launch_bounds__(kBulkThreads, SB_INJECT_MIN_BLOCKS)
    inject_bulk_kernel(const __grid_constant__ LT L) {
  constexpr int VEC = 16 / (int)sizeof(T);
  extern __shared__ uint8_t bulk_smem_raw[];
  uint8_t *stages = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(bulk_smem_raw) + 127) & ~uintptr_t(127));
  __shared__ uint64_t full[kBulkStages], empty[kBulkStages];
  __shared__ int abort_flag;
  __shared__ int64_t pair_soff[kBulkConsumers];
  __shared__ int32_t run_p0[kBulkConsumers], run_len[kBulkConsumers];
  __shared__ uint8_t pair_ok[kBulkConsumers];
  __shared__ sb_inject_desc s_desc;
  __shared__ int64_t s_first;

  const InjectCommon &C = L.c;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tile = blockIdx.x;
  if (threadIdx.x == 0) {
    s_desc = find_desc(L, tile, s_first);
    for (int i = 0; i < kBulkStages; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], kBulkConsumers / 32);
    }
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  const sb_inject_desc &d = s_desc;
  const sb_inject_params &P = C.p;
  const int D = P.head_dim;
  const int row_bytes = D * (int)sizeof(T);
  const int H = P.n_heads;
  const int ua = (int)((int64_t)blockIdx.y * C.units_per_chunk);
  const int nrow = (int)min((int64_t)C.units_per_chunk, C.n_units - ua);
  const tc::Abort ab{&abort_flag, nullptr};

  // ---- per-pair rows (consumer threads), as inject_kernel ----
  const int tpr = C.tpr;
  const int pl = threadIdx.x / tpr;
  const int slice = threadIdx.x - pl * tpr;
  bool ok = false;
  int64_t sp = 0, tp = 0, soff = 0, doff = 0;
  // when tpr does not divide the block (head_dim 96: 6 threads a pair, 42 pairs), the last
  // threads own no pair; they still take part in every barrier
  if (warp < kBulkConsumers / 32 && pl < C.pairs_per_tile) {
    const int64_t pair = (tile - s_first) * C.pairs_per_tile + pl;
    if (pair < d.n_pairs) {
      sp = load_index(d.src_pos, pair, d.pos_dtype);
      tp = load_index(d.dst_pos, pair, d.pos_dtype);
      const int64_t srow = d.src_row == SB_ROW_AT_PAIR ? pair : (d.src_row == SB_ROW_AT_DST_POS ? tp : sp);
      const int64_t drow = d.dst_row == SB_ROW_AT_PAIR ? pair : (d.dst_row == SB_ROW_AT_SRC_POS ? sp : tp);
      int64_t chk = 0;
      ok = resolve_row(d.src, srow, soff) && resolve_row(d.dst, drow, doff);
      if (ok && (d.flags & SB_DESC_CHECK_SRC_IN_DST)) ok = resolve_row(d.dst, sp, chk);
      if (!ok && blockIdx.y == 0 && slice == 0 && C.err != nullptr) atomicAdd(C.err, 1ull);
    }
    if (slice == 0) {
      pair_ok[pl] = ok ? 1 : 0;
      pair_soff[pl] = soff;
    }
  }
  __syncthreads();

  if (warp == kBulkConsumers / 32) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      // runs of valid pairs whose source rows follow each other in memory
      const bool contig = d.src.stride_pos == D && d.src.stride_dim == 1;
      int n_runs = 0;
      uint32_t tx = 0;
      for (int p = 0; p < C.pairs_per_tile; ++p) {
        if (!pair_ok[p]) continue;
        tx += (uint32_t)row_bytes;
        if (n_runs > 0 && contig && run_p0[n_runs - 1] + run_len[n_runs - 1] == p &&
            pair_soff[p] == pair_soff[run_p0[n_runs - 1]] + (int64_t)run_len[n_runs - 1] * D) {
          ++run_len[n_runs - 1];
        } else {
          run_p0[n_runs] = p;
          run_len[n_runs] = 1;
          ++n_runs;
        }
      }
      int h = ua % H, kvi = (ua / H) % C.n_kv_sel, l = (ua / H) / C.n_kv_sel;
      int issued = 0;
      for (int i = 0; i < nrow; ++i) {
        const int st = i % kBulkStages;
        if (i >= kBulkStages && !tc::mbar_wait(&empty[st], ((i / kBulkStages) - 1) & 1, ab, 1, kBulkWaitCycles))
          break;
        const int kv = C.kv_first + kvi;
        const T *base = layer_base<T>(d.src, l) + kv * d.src.stride_kv + h * d.src.stride_head;
        if (++h == H) {
          h = 0;
          if (++kvi == C.n_kv_sel) {
            kvi = 0;
            ++l;
          }
        }
        tc::mbar_arrive_expect_tx(&full[st], tx);
        uint8_t *stage = stages + (size_t)st * kStageBytes;
        for (int r = 0; r < n_runs; ++r) {
          const T *src = base + pair_soff[run_p0[r]];
          // the copy's alignment rule (16-byte addresses and sizes) holds by the launch's choice
          // of this kernel; a row that broke it is left out and its stage never completes
          if ((reinterpret_cast<uintptr_t>(src) & 15) == 0)
            bulk_load(stage + (size_t)run_p0[r] * row_bytes, src, (uint32_t)(run_len[r] * row_bytes), &full[st]);
        }
        ++issued;
      }
      // the copies in flight land before the CTA can exit (only an abort leaves any)
      const int from = issued > kBulkStages ? issued - kBulkStages : 0;
      volatile int never = 0;
      const tc::Abort drain{&never, nullptr};
      for (int i = from; i < issued; ++i)
        tc::mbar_wait(&full[i % kBulkStages], (i / kBulkStages) & 1, drain, 0, kBulkWaitCycles);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const bool neox = P.rotary_style == SB_ROTARY_NEOX;
  int oa, ob;
  if (neox) {
    oa = slice * VEC;
    ob = D / 2 + slice * VEC;
  } else {
    oa = 2 * slice * VEC;
    ob = oa + VEC;
  }
  const bool rot = P.k_angle != SB_ANGLE_NONE && (P.kv_select & SB_KV_K);
  float c1[VEC], s1[VEC], c2[NOPE ? VEC : 1], s2[NOPE ? VEC : 1];
#pragma unroll
  for (int e = 0; e < VEC; ++e) c1[e] = 1.f, s1[e] = 0.f;
#pragma unroll
  for (int e = 0; e < (NOPE ? VEC : 1); ++e) c2[e] = 1.f, s2[e] = 0.f;
  if (rot) {  // the consumers' barriers of the table (the producer warp has left)
    float m1 = 0.f, m2 = 0.f;
    if (ok) pair_angles(P, sp, tp, m1, m2);
    tile_angles<VEC, NOPE, true>(P, C.pairs_per_tile, pl, slice, ok, m1, m2, c1, s1, c2, s2);
  }
  int h = ua % H, kvi = (ua / H) % C.n_kv_sel, l = (ua / H) / C.n_kv_sel;
  bool stalled = false;
#pragma unroll 1
  for (int i = 0; i < nrow; ++i) {
    const int st = i % kBulkStages;
    if (!tc::mbar_wait(&full[st], (i / kBulkStages) & 1, ab, 2, kBulkWaitCycles)) {
      stalled = true;
      break;
    }
    const int kv = C.kv_first + kvi;
    if (ok) {
      const uint8_t *row = stages + (size_t)st * kStageBytes + (size_t)pl * row_bytes;
      Vec<T, VEC> va, vb;
      va = *reinterpret_cast<const Vec<T, VEC> *>(row + oa * (int)sizeof(T));
      vb = *reinterpret_cast<const Vec<T, VEC> *>(row + ob * (int)sizeof(T));
      if (rot && kv == 0) rotate_vectors<T, VEC, NOPE>(va, vb, neox, c1, s1, c2, s2);
      T *t = layer_base<T>(d.dst, l) + kv * d.dst.stride_kv + h * d.dst.stride_head + doff;
      store_vec(t + oa, va);
      store_vec(t + ob, vb);
    }
    if (++h == H) {
      h = 0;
      if (++kvi == C.n_kv_sel) {
        kvi = 0;
        ++l;
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[st]);
  }
  if (stalled && ok && slice == 0 && C.err != nullptr) atomicAdd(C.err, 1ull);
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

bool rows_valid(const sb_rows &r) {
  if (r.base == nullptr && r.layer_ptrs == nullptr) return false;
  if (r.n_logical < 0) return false;
  if (r.block_table != nullptr) {
    if (r.block_size <= 0 || r.n_physical < 0) return false;
    if (r.block_table_dtype != SB_INDEX_I32 && r.block_table_dtype != SB_INDEX_I64) return false;
  }
  return true;
}

// Largest vector width (elements) usable for every descriptor.
int pick_vec(const sb_inject_desc *descs, int n, int D, int es) {
  for (int vec = 16 / es; vec >= 2; vec /= 2) {
    if (D % (2 * vec) != 0) continue;
    bool ok = true;
    const int64_t vb = (int64_t)vec * es;
    for (int i = 0; i < n && ok; ++i) {
      if (descs[i].n_pairs == 0) continue;
      for (const sb_rows *r : {&descs[i].src, &descs[i].dst}) {
        if (r->stride_dim != 1) ok = false;
        if (r->layer_ptrs == nullptr && r->stride_layer % vec) ok = false;
        if (r->block_table != nullptr && r->stride_block % vec) ok = false;
        if (r->stride_kv % vec || r->stride_head % vec || r->stride_pos % vec) ok = false;
        if (r->base != nullptr && (reinterpret_cast<uintptr_t>(r->base) % vb)) ok = false;
      }
    }
    if (ok) return vec;
  }
  return 1;
}

template <typename T, int VEC, typename LT>
int launch_typed(const LT &L, dim3 grid, cudaStream_t st) {
  const bool nope = L.c.p.k_angle == SB_ANGLE_NOPE && (L.c.p.kv_select & SB_KV_K);
  const bool bulk = (L.c.p.flags & SB_INJECT_BULK_STAGED) && VEC * (int)sizeof(T) == 16;
  if (bulk) {
    // the stage ring plus the static tables exceed 48 KB: opt in once per kernel and device
    const void *fn = nope ? (const void *)inject_bulk_kernel<T, LT, true> : (const void *)inject_bulk_kernel<T, LT, false>;
    const int s = ensure_dynamic_smem(fn, (int)kBulkDynSmem);
    if (s != SB_OK) return s;
  }
  const int slot = prof_before(st);
  if (bulk) {
    if (nope)
      inject_bulk_kernel<T, LT, true><<<grid, kBulkThreads, kBulkDynSmem, st>>>(L);
    else
      inject_bulk_kernel<T, LT, false><<<grid, kBulkThreads, kBulkDynSmem, st>>>(L);
  } else if (nope) {
    inject_kernel<T, VEC, LT, true><<<grid, kThreads, 0, st>>>(L);
  } else {
    inject_kernel<T, VEC, LT, false><<<grid, kThreads, 0, st>>>(L);
  }
  prof_after(slot, st);
  return launch_status();
}

template <typename LT>
int launch(const LT &L, int vec, dim3 grid, cudaStream_t st) {
  switch (L.c.p.dtype) {
    case SB_DTYPE_F32:
      if (vec == 4) return launch_typed<float, 4>(L, grid, st);
      if (vec == 2) return launch_typed<float, 2>(L, grid, st);
      return launch_typed<float, 1>(L, grid, st);
    case SB_DTYPE_F16:
      if (vec == 8) return launch_typed<__half, 8>(L, grid, st);
      if (vec == 4) return launch_typed<__half, 4>(L, grid, st);
      if (vec == 2) return launch_typed<__half, 2>(L, grid, st);
      return launch_typed<__half, 1>(L, grid, st);
    case SB_DTYPE_BF16:
      if (vec == 8) return launch_typed<__nv_bfloat16, 8>(L, grid, st);
      if (vec == 4) return launch_typed<__nv_bfloat16, 4>(L, grid, st);
      if (vec == 2) return launch_typed<__nv_bfloat16, 2>(L, grid, st);
      return launch_typed<__nv_bfloat16, 1>(L, grid, st);
  }
  return SB_ERR_UNSUPPORTED;
}

int validate_params(const sb_inject_params *p) {
  if (p == nullptr) return SB_ERR_INVALID_ARGUMENT;
  if (p->n_layers <= 0 || p->n_heads <= 0) return SB_ERR_INVALID_ARGUMENT;
  if (p->head_dim < 2 || p->head_dim % 2 || p->head_dim > 512) return SB_ERR_UNSUPPORTED;
  if (elem_bytes(p->dtype) == 0) return SB_ERR_UNSUPPORTED;
  if (p->rotary_style != SB_ROTARY_INTERLEAVED && p->rotary_style != SB_ROTARY_NEOX)
    return SB_ERR_INVALID_ARGUMENT;
  if (p->k_angle < SB_ANGLE_NONE || p->k_angle > SB_ANGLE_CONST) return SB_ERR_INVALID_ARGUMENT;
  if (p->kv_select < 1 || p->kv_select > 3) return SB_ERR_INVALID_ARGUMENT;
  if (p->flags & ~SB_INJECT_BULK_STAGED) return SB_ERR_INVALID_ARGUMENT;
  if (p->k_angle != SB_ANGLE_NONE && (p->kv_select & SB_KV_K) && p->inv_freq == nullptr)
    return SB_ERR_INVALID_ARGUMENT;
  return SB_OK;
}

// Launch geometry shared by both descriptor-table forms: the common fields,
// each descriptor's first pair tile (tile_start[n_desc + 1]) and the grid.
// Returns SB_OK with grid.x == 0 when there is nothing to do.
int plan_inject(const sb_inject_desc *descs, int n_desc, const sb_inject_params *params, uint64_t *err,
                InjectCommon &C, int64_t *tile_start, int &vec, dim3 &grid) {
  memset(&C, 0, sizeof(C));
  C.p = *params;
  C.err = reinterpret_cast<unsigned long long *>(err);
  C.n_desc = n_desc;
  const int D = params->head_dim;
  const int es = elem_bytes(params->dtype);
  vec = pick_vec(descs, n_desc, D, es);
  C.tpr = D / (2 * vec);
  if (C.tpr > kThreads) return SB_ERR_UNSUPPORTED;
  C.pairs_per_tile = kThreads / C.tpr;
  C.n_kv_sel = params->kv_select == SB_KV_BOTH ? 2 : 1;
  C.kv_first = params->kv_select == SB_KV_V ? 1 : 0;
  C.n_units = (int64_t)params->n_layers * C.n_kv_sel * params->n_heads;
  if (C.n_units > 0x7fffffffLL) return SB_ERR_TOO_LARGE;  // the kernel counts units in int32
  int64_t tiles = 0;
  for (int i = 0; i < n_desc; ++i) {
    tile_start[i] = tiles;
    tiles += (descs[i].n_pairs + C.pairs_per_tile - 1) / C.pairs_per_tile;
  }
  tile_start[n_desc] = tiles;
  grid = dim3(0, 1);
  if (tiles == 0) return SB_OK;
  if (tiles > 0x7fffffffLL) return SB_ERR_TOO_LARGE;
  // Aim for ~16 waves of resident CTAs so the last wave's imbalance is small,
  // while keeping at least 8 rows per thread to amortise the cos/sin set-up.
  // A launch with fewer pair tiles than two waves of resident CTAs (one
  // layer of a few thousand pairs) would leave SMs idle at 8 rows per thread:
  // there the units are split into as many chunks as fit in one wave, down
  // to the rows a thread keeps in flight at once.
  const int64_t slots = (int64_t)sm_count() * SB_INJECT_MIN_BLOCKS;
  int64_t chunks;
  if (tiles >= 2 * slots) {
    const int64_t target = (int64_t)sm_count() * (2048 / kThreads) * SB_INJECT_TARGET_WAVES;
    chunks = std::max<int64_t>(1, (target + tiles - 1) / tiles);
    chunks = std::min<int64_t>(chunks, std::max<int64_t>(1, C.n_units / SB_INJECT_MIN_ROWS));
  } else {
    chunks = std::max<int64_t>(1, slots / tiles);
    chunks = std::min<int64_t>(chunks, std::max<int64_t>(1, (C.n_units + kUnroll - 1) / kUnroll));
  }
  chunks = std::min<int64_t>(chunks, 65535);
  int64_t upc = (C.n_units + chunks - 1) / chunks;
  chunks = (C.n_units + upc - 1) / upc;
  if (upc > 0x7fffffffLL) return SB_ERR_TOO_LARGE;
  C.units_per_chunk = (int32_t)upc;
  grid = dim3((unsigned)tiles, (unsigned)chunks);
  return SB_OK;
}

template <int MAXD>
int inject_impl(const sb_inject_desc *descs, int n_desc, const sb_inject_params *params,
                uint64_t *err, cudaStream_t st) {
  InjectLaunch<MAXD> L;
  memset(&L, 0, sizeof(L));
  int vec = 1;
  dim3 grid;
  const int s = plan_inject(descs, n_desc, params, err, L.c, L.tile_start, vec, grid);
  if (s != SB_OK || grid.x == 0) return s;
  for (int i = 0; i < n_desc; ++i) L.desc[i] = descs[i];
  return launch(L, vec, grid, st);
}

int validate_descs(const sb_inject_desc *descs, int32_t n_desc) {
  if (n_desc == 0) return SB_OK;
  if (descs == nullptr) return SB_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < n_desc; ++i) {
    const sb_inject_desc &d = descs[i];
    if (d.n_pairs < 0) return SB_ERR_INVALID_ARGUMENT;
    if (d.n_pairs == 0) continue;
    if (d.src_pos == nullptr || d.dst_pos == nullptr) return SB_ERR_INVALID_ARGUMENT;
    if (d.pos_dtype != SB_INDEX_I32 && d.pos_dtype != SB_INDEX_I64) return SB_ERR_INVALID_ARGUMENT;
    if (d.src_row < SB_ROW_AT_SRC_POS || d.src_row > SB_ROW_AT_PAIR) return SB_ERR_INVALID_ARGUMENT;
    if (d.dst_row < SB_ROW_AT_SRC_POS || d.dst_row > SB_ROW_AT_PAIR) return SB_ERR_INVALID_ARGUMENT;
    if (!rows_valid(d.src) || !rows_valid(d.dst)) return SB_ERR_INVALID_ARGUMENT;
  }
  return SB_OK;
}

}  // namespace

int64_t inject_table_bytes(int32_t n_desc) {
  if (n_desc < 0) return SB_ERR_INVALID_ARGUMENT;
  const int64_t d = (int64_t)n_desc * (int64_t)sizeof(sb_inject_desc);
  return (d + 15) / 16 * 16 + ((int64_t)n_desc + 1) * 8;
}

int inject_dispatch(const sb_inject_desc *descs, int32_t n_desc, const sb_inject_params *params,
                    uint64_t *err_counter, cudaStream_t st) {
  int s = validate_params(params);
  if (s != SB_OK) return s;
  if (n_desc < 0 || n_desc > SB_MAX_INJECT_DESC) return SB_ERR_INVALID_ARGUMENT;
  if (n_desc == 0) return SB_OK;
  s = validate_descs(descs, n_desc);
  if (s != SB_OK) return s;
  if (n_desc == 1) return inject_impl<1>(descs, n_desc, params, err_counter, st);
  return inject_impl<SB_MAX_INJECT_DESC>(descs, n_desc, params, err_counter, st);
}

// Any number of descriptors in one launch: the table (descriptors, then each
// descriptor's first pair tile) is staged on the host and copied to `table`
// on the stream ahead of the kernel.
int inject_table_dispatch(const sb_inject_desc *descs, int32_t n_desc, const sb_inject_params *params,
                          void *table, int64_t table_bytes, uint64_t *err_counter, cudaStream_t st) {
  int s = validate_params(params);
  if (s != SB_OK) return s;
  if (n_desc < 0 || n_desc > (1 << 24)) return SB_ERR_INVALID_ARGUMENT;
  if (n_desc == 0) return SB_OK;
  s = validate_descs(descs, n_desc);
  if (s != SB_OK) return s;
  const int64_t need = inject_table_bytes(n_desc);
  if (table == nullptr || table_bytes < need) return SB_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(table) % 16) return SB_ERR_INVALID_ARGUMENT;
  const int64_t desc_bytes = (int64_t)n_desc * (int64_t)sizeof(sb_inject_desc);
  const int64_t ts_off = (desc_bytes + 15) / 16 * 16;
  std::vector<uint8_t> host((size_t)need, 0);
  memcpy(host.data(), descs, (size_t)desc_bytes);
  int64_t *tile_start = reinterpret_cast<int64_t *>(host.data() + ts_off);
  InjectLaunchTable L;
  memset(&L, 0, sizeof(L));
  int vec = 1;
  dim3 grid;
  s = plan_inject(descs, n_desc, params, err_counter, L.c, tile_start, vec, grid);
  if (s != SB_OK || grid.x == 0) return s;
  uint8_t *dev = static_cast<uint8_t *>(table);
  // pageable source: staged before this call returns, so `host` may go out of scope
  const cudaError_t e = cudaMemcpyAsync(dev, host.data(), (size_t)need, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SB_ERR_CUDA;
  }
  L.desc = reinterpret_cast<const sb_inject_desc *>(dev);
  L.tile_start = reinterpret_cast<const int64_t *>(dev + ts_off);
  return launch(L, vec, grid, st);
}

}  // namespace sb

extern "C" SB_API int sb_inject(const sb_inject_desc *descs, int32_t n_desc,
                                const sb_inject_params *params, uint64_t *err_counter,
                                void *stream) {
  return sb::inject_dispatch(descs, n_desc, params, err_counter,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" SB_API int64_t sb_inject_table_bytes(int32_t n_desc) { return sb::inject_table_bytes(n_desc); }

extern "C" SB_API int sb_inject_many(const sb_inject_desc *descs, int32_t n_desc, const sb_inject_params *params,
                                     void *table, int64_t table_bytes, uint64_t *err_counter, void *stream) {
  return sb::inject_table_dispatch(descs, n_desc, params, table, table_bytes, err_counter,
                                   reinterpret_cast<cudaStream_t>(stream));
}

extern "C" SB_API int64_t sb_permute_workspace_bytes(int64_t n_pairs, int32_t n_layers,
                                                     int32_t n_heads, int32_t head_dim,
                                                     int32_t dtype) {
  const int es = sb::elem_bytes(dtype);
  if (es == 0 || n_pairs < 0 || n_layers <= 0 || n_heads <= 0 || head_dim <= 0) return -1;
  // n_pairs * n_layers * 2 * n_heads * head_dim * es, rejected (-1) if it overflows int64
  int64_t b = n_pairs;
  for (const int64_t f : {(int64_t)n_layers, (int64_t)2, (int64_t)n_heads, (int64_t)head_dim, (int64_t)es})
    if (__builtin_mul_overflow(b, f, &b)) return -1;
  return b;
}

extern "C" SB_API int sb_permute_paged(const sb_rows *cache, const void *src_pos,
                                       const void *dst_pos, int64_t n_pairs, int32_t pos_dtype,
                                       const sb_inject_params *params, void *workspace,
                                       int64_t workspace_bytes, uint64_t *err_counter,
                                       void *stream) {
  if (cache == nullptr || params == nullptr) return SB_ERR_INVALID_ARGUMENT;
  if (params->k_angle == SB_ANGLE_CONST) return SB_ERR_INVALID_ARGUMENT;
  if (n_pairs < 0) return SB_ERR_INVALID_ARGUMENT;
  if (n_pairs == 0) return SB_OK;
  const int64_t need = sb_permute_workspace_bytes(n_pairs, params->n_layers, params->n_heads,
                                                  params->head_dim, params->dtype);
  if (need < 0) return SB_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < need) return SB_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return SB_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t H = params->n_heads, D = params->head_dim;

  sb_rows ws;
  memset(&ws, 0, sizeof(ws));
  ws.base = workspace;
  ws.stride_dim = 1;
  ws.stride_head = D;
  ws.stride_kv = H * D;
  ws.stride_pos = 2 * H * D;
  ws.stride_layer = n_pairs * 2 * H * D;
  ws.n_logical = n_pairs;

  // Phase 1: snapshot every source row (plain copy, uncounted).
  sb_inject_desc g;
  memset(&g, 0, sizeof(g));
  g.src = *cache;
  g.dst = ws;
  g.src_pos = src_pos;
  g.dst_pos = dst_pos;
  g.n_pairs = n_pairs;
  g.pos_dtype = pos_dtype;
  g.src_row = SB_ROW_AT_SRC_POS;
  g.dst_row = SB_ROW_AT_PAIR;
  sb_inject_params gp = *params;
  gp.k_angle = SB_ANGLE_NONE;
  int s = sb::inject_dispatch(&g, 1, &gp, nullptr, st);
  if (s != SB_OK) return s;

  // Phase 2: write the snapshot to the destinations, rotating K.  Pairs whose
  // source row was out of range (left unsnapshotted) are skipped and counted.
  sb_inject_desc w = g;
  w.src = ws;
  w.dst = *cache;
  w.src_row = SB_ROW_AT_PAIR;
  w.dst_row = SB_ROW_AT_DST_POS;
  w.flags = SB_DESC_CHECK_SRC_IN_DST;
  return sb::inject_dispatch(&w, 1, params, err_counter, st);
}

// ---------------------------------------------------------------------------
// In-place permutation without any allocation.
//
// Some callers cannot allocate device memory at the moment they permute:
// an inference engine's per-layer hook runs inside the model's forward pass,
// where the engine has pre-sized its memory pool during start-up profiling
// (an allocation there eats into the KV-cache budget or fails) or is capturing
// the step into a CUDA graph; C, Go or Java callers that bind this library
// directly have no caching allocator to borrow scratch space from.  For them
// the source-row snapshot lives in this fixed device array instead of a
// caller-provided workspace.  Every GPU that loads the library holds it until
// the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_permute_scratch[SB_PERMUTE_NOALLOC_SCRATCH_BYTES];

namespace sb {
namespace {
// The array's device address is resolved once per CUDA context.  Contexts are
// told apart by cuCtxGetId, an id the driver never reuses within a process, so
// a context destroyed and created again (cudaDeviceReset) or a driver-API
// context of the caller's own on the same device resolves the address anew.
typedef CUresult (*ctx_get_current_fn)(CUcontext *);
typedef CUresult (*ctx_get_id_fn)(CUcontext, unsigned long long *);
constexpr int kScratchSlots = 64;
std::mutex g_scratch_mu;
unsigned long long g_scratch_ctx[kScratchSlots] = {};  // context id + 1 (0 = empty slot)
void *g_scratch_ptr[kScratchSlots] = {};
int g_scratch_next = 0;

template <typename F>
F driver_fn(const char *name) {
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(p);
}

// The device address of g_permute_scratch in the calling thread's current
// context (the device's primary context if none is current yet).
int scratch_address(void **out) {
  static ctx_get_current_fn get_current = driver_fn<ctx_get_current_fn>("cuCtxGetCurrent");
  static ctx_get_id_fn get_id = driver_fn<ctx_get_id_fn>("cuCtxGetId");
  if (get_current == nullptr || get_id == nullptr) return SB_ERR_UNSUPPORTED;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return SB_ERR_CUDA;
  void *p = nullptr;
  cudaError_t e = cudaSuccess;
  if (ctx == nullptr) {
    // no context current yet: this runtime call makes the device's primary context current
    e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      set_last_cuda_error(e);
      return SB_ERR_CUDA;
    }
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return SB_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  for (int i = 0; i < kScratchSlots; ++i) {
    if (g_scratch_ctx[i] == id + 1) {
      *out = g_scratch_ptr[i];
      return SB_OK;
    }
  }
  if (p == nullptr) {
    // first call in this context: the host-side symbol is only a stand-in and must never reach a kernel
    e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_cuda_error(e);
      return SB_ERR_CUDA;
    }
  }
  g_scratch_ctx[g_scratch_next] = id + 1;
  g_scratch_ptr[g_scratch_next] = p;
  g_scratch_next = (g_scratch_next + 1) % kScratchSlots;
  *out = p;
  return SB_OK;
}
}  // namespace
}  // namespace sb

extern "C" SB_API int sb_permute_paged_noalloc(const sb_rows *cache, const void *src_pos, const void *dst_pos,
                                               int64_t n_pairs, int32_t pos_dtype, const sb_inject_params *params,
                                               uint64_t *err_counter, void *stream) {
  if (cache == nullptr || params == nullptr || n_pairs < 0) return SB_ERR_INVALID_ARGUMENT;
  if (n_pairs == 0) return SB_OK;
  const int64_t need = sb_permute_workspace_bytes(n_pairs, params->n_layers, params->n_heads, params->head_dim,
                                                  params->dtype);
  if (need < 0) return SB_ERR_INVALID_ARGUMENT;
  if (need > SB_PERMUTE_NOALLOC_SCRATCH_BYTES) return SB_ERR_TOO_LARGE;
  void *scratch = nullptr;
  const int s = sb::scratch_address(&scratch);
  if (s != SB_OK) return s;
  // Rows are snapshotted for every pair before any is read back, and pairs
  // whose source was out of range are skipped rather than read, so the
  // scratch needs no clearing between calls.
  return sb_permute_paged(cache, src_pos, dst_pos, n_pairs, pos_dtype, params, scratch,
                          SB_PERMUTE_NOALLOC_SCRATCH_BYTES, err_counter, stream);
}

/* A C caller of the library, without Python or torch: one paged copy inject
 * (flat donor rows -> a [nb, 2, H, bs, D] bf16 cache through a block table),
 * checked bit for bit on the host, plus the status of an invalid call.
 * Built and run by tests/test_c_abi_gpu.py; exits 0 on success. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "semblend_b200.h"

#define H 2
#define D 64
#define BS 16
#define NB 12
#define SD 100
#define NP 40

#define CHECK(x)                                                              \
  do {                                                                        \
    cudaError_t e_ = (x);                                                     \
    if (e_ != cudaSuccess) {                                                  \
      fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                \
      return 2;                                                               \
    }                                                                         \
  } while (0)

int main(void) {
  const size_t donor_n = (size_t)2 * H * SD * D, cache_n = (size_t)NB * 2 * H * BS * D;
  uint16_t *donor = malloc(donor_n * 2), *cache = malloc(cache_n * 2), *want = malloc(cache_n * 2);
  int32_t bt[4] = {7, 2, 10, 5}, dpos[NP], tpos[NP];
  uint64_t skipped = 0;
  for (size_t i = 0; i < donor_n; ++i) donor[i] = (uint16_t)(0x3c00 + (i * 2654435761u >> 20) % 1024);
  for (size_t i = 0; i < cache_n; ++i) cache[i] = (uint16_t)(i * 40503u);
  memcpy(want, cache, cache_n * 2);
  for (int i = 0; i < NP; ++i) {
    dpos[i] = (i * 7) % SD;
    tpos[i] = (i * 5 + 3) % (4 * BS); /* distinct targets: 5 is coprime with 64 */
  }
  /* host model of the copy: donor [2, H, SD, D] -> cache[bt[t / BS], kv, h, t % BS, :] */
  for (int i = 0; i < NP; ++i)
    for (int kv = 0; kv < 2; ++kv)
      for (int h = 0; h < H; ++h) {
        const size_t src = (((size_t)kv * H + h) * SD + dpos[i]) * D;
        const size_t dst = ((((size_t)bt[tpos[i] / BS] * 2 + kv) * H + h) * BS + tpos[i] % BS) * D;
        memcpy(want + dst, donor + src, D * 2);
      }

  void *d_donor, *d_cache, *d_bt, *d_dpos, *d_tpos, *d_err;
  CHECK(cudaMalloc(&d_donor, donor_n * 2));
  CHECK(cudaMalloc(&d_cache, cache_n * 2));
  CHECK(cudaMalloc(&d_bt, sizeof bt));
  CHECK(cudaMalloc(&d_dpos, sizeof dpos));
  CHECK(cudaMalloc(&d_tpos, sizeof tpos));
  CHECK(cudaMalloc(&d_err, 8));
  CHECK(cudaMemcpy(d_donor, donor, donor_n * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_cache, cache, cache_n * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_bt, bt, sizeof bt, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_dpos, dpos, sizeof dpos, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_tpos, tpos, sizeof tpos, cudaMemcpyHostToDevice));
  CHECK(cudaMemset(d_err, 0, 8));

  sb_rows src, dst;
  memset(&src, 0, sizeof src);
  memset(&dst, 0, sizeof dst);
  src.base = d_donor;
  src.stride_kv = (int64_t)H * SD * D;
  src.stride_head = (int64_t)SD * D;
  src.stride_pos = D;
  src.stride_dim = 1;
  src.n_logical = SD;
  dst.base = d_cache;
  dst.stride_block = (int64_t)2 * H * BS * D;
  dst.stride_kv = (int64_t)H * BS * D;
  dst.stride_head = (int64_t)BS * D;
  dst.stride_pos = D;
  dst.stride_dim = 1;
  dst.block_table = d_bt;
  dst.n_logical = 4;
  dst.n_physical = NB;
  dst.block_size = BS;
  dst.block_table_dtype = SB_INDEX_I32;
  sb_inject_desc desc;
  memset(&desc, 0, sizeof desc);
  desc.src = src;
  desc.dst = dst;
  desc.src_pos = d_dpos;
  desc.dst_pos = d_tpos;
  desc.n_pairs = NP;
  desc.pos_dtype = SB_INDEX_I32;
  desc.src_row = SB_ROW_AT_SRC_POS;
  desc.dst_row = SB_ROW_AT_DST_POS;
  sb_inject_params p;
  memset(&p, 0, sizeof p);
  p.n_layers = 1;
  p.n_heads = H;
  p.head_dim = D;
  p.dtype = SB_DTYPE_BF16;
  p.rotary_style = SB_ROTARY_NEOX;
  p.k_angle = SB_ANGLE_NONE;
  p.kv_select = SB_KV_BOTH;

  int s = sb_inject(&desc, 1, &p, (uint64_t *)d_err, NULL);
  if (s != SB_OK) {
    fprintf(stderr, "sb_inject: %s\n", sb_status_string(s));
    return 1;
  }
  CHECK(cudaDeviceSynchronize());
  CHECK(cudaMemcpy(cache, d_cache, cache_n * 2, cudaMemcpyDeviceToHost));
  CHECK(cudaMemcpy(&skipped, d_err, 8, cudaMemcpyDeviceToHost));
  if (memcmp(cache, want, cache_n * 2) != 0 || skipped != 0) {
    fprintf(stderr, "cache differs from the host copy (skipped %llu)\n", (unsigned long long)skipped);
    return 1;
  }
  /* an invalid call launches nothing and says why */
  s = sb_inject(&desc, -1, &p, (uint64_t *)d_err, NULL);
  if (s != SB_ERR_INVALID_ARGUMENT) {
    fprintf(stderr, "expected SB_ERR_INVALID_ARGUMENT, got %d\n", s);
    return 1;
  }
  printf("c abi ok: %d pairs copied; invalid call -> %s\n", NP, sb_status_string(s));
  cudaFree(d_donor);
  cudaFree(d_cache);
  cudaFree(d_bt);
  cudaFree(d_dpos);
  cudaFree(d_tpos);
  cudaFree(d_err);
  free(donor);
  free(cache);
  free(want);
  return 0;
}

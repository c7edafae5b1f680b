/*
 * semblend_b200 — C ABI of the B200-native donor-reuse hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * and an opaque CUDA stream handle (a cudaStream_t passed as void*).  Nothing
 * here allocates device memory: scratch space is passed in by the caller and
 * sized by the matching *_workspace_bytes() query.  Calls are asynchronous on
 * the given stream.  A return value of SB_OK means the work was enqueued;
 * negative values mean the arguments were rejected and nothing was launched.
 *
 * The reference implementation (SemBlend 0.3.2) is pure Python + Triton; the
 * interfaces each entry point replaces are cited by file:line of that project.
 */
#ifndef SEMBLEND_B200_H
#define SEMBLEND_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Status codes                                                              */
/* ------------------------------------------------------------------------ */
#define SB_OK 0
#define SB_ERR_INVALID_ARGUMENT (-1)
#define SB_ERR_UNSUPPORTED (-2)
#define SB_ERR_CUDA (-3)
#define SB_ERR_WORKSPACE_TOO_SMALL (-4)
#define SB_ERR_TOO_LARGE (-5)

/* Element types. */
#define SB_DTYPE_F32 0
#define SB_DTYPE_F16 1
#define SB_DTYPE_BF16 2

/* Index types (positions, block tables). */
#define SB_INDEX_I32 0
#define SB_INDEX_I64 1

/* RoPE pairing: interleaved pairs (2i, 2i+1) as the reference rotates them,
 * or neox half-rotation pairs (i, i + D/2). */
#define SB_ROTARY_INTERLEAVED 0
#define SB_ROTARY_NEOX 1

/* Angle applied to K rows. */
#define SB_ANGLE_NONE 0  /* plain copy                                     */
#define SB_ANGLE_DELTA 1 /* rotate by (dst_pos - src_pos) * inv_freq          */
#define SB_ANGLE_NOPE 2  /* rotate by -src_pos, then by +dst_pos (two steps)  */
#define SB_ANGLE_CONST 3 /* rotate by const_delta * inv_freq                  */

/* Which position selects a source / destination row. */
#define SB_ROW_AT_SRC_POS 0
#define SB_ROW_AT_DST_POS 1
#define SB_ROW_AT_PAIR 2 /* row index = pair index (a per-pair snapshot)     */

/* Row selection: bit 0 = K rows (kv index 0), bit 1 = V rows (kv index 1). */
#define SB_KV_K 1
#define SB_KV_V 2
#define SB_KV_BOTH 3

/* Maximum descriptors a single sb_inject call accepts. */
#define SB_MAX_INJECT_DESC 64

/* ------------------------------------------------------------------------ */
/* Row addressing                                                           */
/* ------------------------------------------------------------------------ */
/* A set of KV rows of head_dim elements.  The element (layer l, kv, head h,
 * position p, dim d) lives at
 *     layer_base(l) + kv*stride_kv + h*stride_head + row_offset(p) + d*stride_dim
 * (element units), where layer_base(l) = layer_ptrs[l] if layer_ptrs != NULL
 * (a DEVICE array of n_layers byte addresses, each 16-byte aligned) else
 * base + l*stride_layer.
 *
 * Flat rows (block_table == NULL): row_offset(p) = p*stride_pos and positions
 * p outside [0, n_logical) are out of range.
 * Paged rows: lb = p / block_size must lie in [0, n_logical) (the block-table
 * length), phys = block_table[lb] must lie in [0, n_physical), and
 * row_offset(p) = phys*stride_block + (p % block_size)*stride_pos.
 * These strides cover the reference layout [nb, 2, H, bs, D], vLLM's
 * FlashAttention layout [2, nb, bs, H, D] and TRT-LLM's [nb, 2, bs, H, D]. */
typedef struct sb_rows {
  void *base;
  const uint64_t *layer_ptrs;
  int64_t stride_layer, stride_block, stride_kv, stride_head, stride_pos,
      stride_dim;
  const void *block_table;
  int64_t n_logical;
  int64_t n_physical;
  int32_t block_size;
  int32_t block_table_dtype; /* SB_INDEX_I32 or SB_INDEX_I64 */
} sb_rows;

/* One independent inject job: a pair list moving rows from src to dst. */
typedef struct sb_inject_desc {
  sb_rows src;
  sb_rows dst;
  const void *src_pos; /* device, n_pairs entries */
  const void *dst_pos; /* device, n_pairs entries */
  int64_t n_pairs;
  int32_t pos_dtype; /* SB_INDEX_I32 or SB_INDEX_I64 */
  int32_t src_row;   /* SB_ROW_AT_SRC_POS or SB_ROW_AT_PAIR */
  int32_t dst_row;   /* SB_ROW_AT_DST_POS, SB_ROW_AT_SRC_POS or SB_ROW_AT_PAIR */
  int32_t flags;     /* SB_DESC_* bits */
} sb_inject_desc;

/* Also require src_pos to address a valid row of dst (used when the source
 * rows were snapshotted out of dst and are read back by pair index). */
#define SB_DESC_CHECK_SRC_IN_DST 1

/* sb_inject_params.flags: stage the source rows in shared memory through
 * 1-D bulk copies (cp.async.bulk, one per run of contiguous rows, a 3-stage
 * ring per CTA) instead of direct 16-byte loads.  Applies when every row is a
 * whole number of 16-byte vectors at 16-byte aligned addresses (otherwise the
 * direct path runs); same results.  Off by default: on B200 the direct path
 * is faster on the reference's workloads except for whole-chunk reuse (see
 * the bench's A/B). */
#define SB_INJECT_BULK_STAGED 1

/* Parameters shared by every descriptor of one call. */
typedef struct sb_inject_params {
  int32_t n_layers;
  int32_t n_heads;
  int32_t head_dim;     /* even, <= 512 */
  int32_t dtype;        /* element type of both src and dst rows */
  int32_t rotary_style; /* SB_ROTARY_* */
  int32_t k_angle;      /* SB_ANGLE_* for K rows; V rows are always copied */
  int32_t kv_select;    /* SB_KV_* */
  int32_t flags;        /* SB_INJECT_* bits (0: the default path) */
  int64_t const_delta;    /* for SB_ANGLE_CONST */
  const float *inv_freq;  /* device, head_dim/2 floats; unused for SB_ANGLE_NONE */
} sb_inject_params;

/* Fused donor-KV gather + RoPE correction of K + scatter (paged or flat).
 *
 * For each descriptor, pair i and every (layer, kv, head) row selected by
 * kv_select: read the source row, rotate it in fp32 when it is a K row and
 * k_angle != SB_ANGLE_NONE (rounding each product and sum separately, as the
 * reference's torch expressions do), and store it in the element type at the
 * destination row.  A pair whose source or destination row is out of range is
 * skipped and counted once in *err_counter (a device uint64, may be NULL),
 * the way the reference's GPU kernels skip them.  Pairs of one call must not
 * write the same destination row twice, and destination rows must not be the
 * source rows of other pairs (use sb_permute_paged for in-place permutations).
 *
 * Replaces:
 *   rope_correct_scatter_paged   semblend_core/rope_correction.py:193-282
 *   scatter_donor_kv             semblend_core/triton_kernels.py:132-191
 *   scatter_donor_kv_paged       semblend_core/triton_kernels.py:279-356
 *   rope_correct_k               semblend_core/rope_correction.py:336-399
 *   apply_rope_delta_inplace     semblend_core/rope_correction.py:699-783
 * (the Triton kernels at triton_kernels.py:60-129, :201-276 and
 *  rope_correction.py:69-190). */
SB_API int sb_inject(const sb_inject_desc *descs, int32_t n_desc,
                     const sb_inject_params *params, uint64_t *err_counter,
                     void *stream);

/* Device bytes of the descriptor table sb_inject_many needs for n_desc
 * descriptors. */
SB_API int64_t sb_inject_table_bytes(int32_t n_desc);

/* sb_inject for any number of descriptors (every request of a step) in one
 * launch: the descriptors and each one's first pair tile are copied on the
 * stream into `table` (device memory, 16-byte aligned, table_bytes >=
 * sb_inject_table_bytes(n_desc)), which the kernel reads; the table must not
 * be written again until this launch has run (stream order).  Same
 * arguments, semantics and replaced reference functions as sb_inject. */
SB_API int sb_inject_many(const sb_inject_desc *descs, int32_t n_desc,
                          const sb_inject_params *params, void *table, int64_t table_bytes,
                          uint64_t *err_counter, void *stream);

/* Bytes of workspace sb_permute_paged needs for n_pairs pairs; -1 for an
 * invalid argument or a size that overflows int64. */
SB_API int64_t sb_permute_workspace_bytes(int64_t n_pairs, int32_t n_layers,
                                          int32_t n_heads, int32_t head_dim,
                                          int32_t dtype);

/* In-place permutation of rows inside one (paged or flat) cache: every source
 * row (K and V, all layers and heads) is first copied into the workspace, then
 * written to its destination with K rotated by k_angle (SB_ANGLE_DELTA or
 * SB_ANGLE_NOPE; SB_ANGLE_NONE copies).  Sources may overlap destinations.
 *
 * Replaces:
 *   permute_paged_kv_with_rope   semblend_core/rope_correction.py:407-476
 *   nope_permute_paged_kv        semblend_core/rope_correction.py:599-696
 *   (and _nope_permute_paged_kernel, rope_correction.py:499-596) */
SB_API int sb_permute_paged(const sb_rows *cache, const void *src_pos,
                            const void *dst_pos, int64_t n_pairs,
                            int32_t pos_dtype, const sb_inject_params *params,
                            void *workspace, int64_t workspace_bytes,
                            uint64_t *err_counter, void *stream);

/* Size of the fixed device scratch array used by sb_permute_paged_noalloc
 * (32 MiB: for example one layer of 16384 pairs x 4 KV heads x head_dim 128
 * in bf16). */
#define SB_PERMUTE_NOALLOC_SCRATCH_BYTES (32LL << 20)

/* sb_permute_paged for callers that cannot allocate device memory when they
 * permute: an engine hook running inside the model's forward pass (whose
 * memory pool was sized at start-up, or which is being captured into a CUDA
 * graph), or a C / Go / Java caller without a caching allocator.  Same
 * arguments and results as sb_permute_paged minus the workspace: the source
 * rows are snapshotted into a fixed SB_PERMUTE_NOALLOC_SCRATCH_BYTES device
 * array inside this library (held on every GPU that loads it until exit).
 * Returns SB_ERR_TOO_LARGE, launching nothing, when
 * sb_permute_workspace_bytes(...) exceeds that size (or overflows).  It
 * allocates nothing.  The first call in each CUDA context (the device's
 * primary context, or a driver-API context current on the calling thread)
 * resolves the array's device address in that context; make that call before
 * any stream capture.  A context destroyed and created again (cudaDeviceReset)
 * counts as a new context.  All calls share the one array, which keeps the
 * last call's rows: calls whose executions overlap on the GPU (other streams,
 * other threads) race on it and must be serialised by the caller.  No
 * counterpart in the reference (its permutation allocates with torch). */
SB_API int sb_permute_paged_noalloc(const sb_rows *cache, const void *src_pos,
                                    const void *dst_pos, int64_t n_pairs, int32_t pos_dtype,
                                    const sb_inject_params *params, uint64_t *err_counter,
                                    void *stream);

/* ------------------------------------------------------------------------ */
/* Donor search                                                             */
/* ------------------------------------------------------------------------ */
/* Refresh the 16-bit screening copy of rows of a row-major fp32 embedding
 * matrix (row pitch ld_emb floats) into emb16 (shadow_dtype SB_DTYPE_F16 or
 * SB_DTYPE_BF16, row pitch ld_16 elements, columns [dim, dim_pad) zeroed),
 * and raise stats[0] / stats[1] (device floats, start at 0) to the largest
 * ||e - e16|| and ||e16|| seen (+inf if a value overflows the 16-bit type).
 * Rows are rows[0..n_rows) (device int64) or, when rows is NULL, the range
 * [row_begin, row_begin + n_rows).  This is the device side of the
 * reference's row write in DonorStore.add_donor
 * (semblend_core/donor_store.py:155-161). */
SB_API int sb_search_prepare_rows(const float *emb, int64_t ld_emb, void *emb16, int64_t ld_16,
                                  int32_t dim, int32_t dim_pad, int32_t shadow_dtype,
                                  const int64_t *rows, int64_t row_begin, int64_t n_rows,
                                  float *stats, void *stream);

/* Workspace bytes sb_cosine_topk needs. */
SB_API int64_t sb_cosine_topk_workspace_bytes(int32_t n_queries, int64_t n_rows, int32_t dim,
                                              int32_t dim_pad, int32_t capacity);

/* Exact brute-force cosine top-k for a batch of queries.
 *
 * For each query q (row of `queries`, pitch ld_q): qn = q / (||q|| + 1e-8)
 * in fp32; returns the k rows j < n_rows with valid[j] != 0 (valid may be
 * NULL) and fp32 similarity emb[j] . qn >= min_similarity, ordered by
 * (similarity desc, j asc), as out_ids[q*k + r] = j + id_offset and
 * out_scores[q*k + r]; missing entries are -1 / -inf.  Screening runs on the
 * tensor cores on the 16-bit copy (emb16 of shadow_dtype, dim_pad a multiple
 * of 64, <= 512) and every candidate within the proven 16-bit error bound is
 * rescored exactly in fp32, so the result equals the fp32 computation.  k <= 32; capacity (>= k) bounds the
 * screening candidates kept per query.  *status (device int32, zeroed by the
 * caller) gets bit 0 set if some query had more than `capacity` candidates
 * (its results are withheld: retry with a larger capacity) and a value >= 2
 * if a kernel wait timed out.  The screening kernel hands out its work units
 * from a counter pair inside the library (one of 64 per device, taken round
 * robin per call and reset by the call's last CTA): at most 64 calls may be in
 * flight on one device at a time, and the first call on a device looks the
 * counters up (make it before any stream capture).
 *
 * Replaces the cosine / threshold / top-k stage of DonorStore.find_donors
 * (semblend_core/donor_store.py:323-341) and DonorStore.find_donor (:205-229),
 * one query at a time there. */
SB_API int sb_cosine_topk(const float *emb, int64_t ld_emb, const void *emb16, int64_t ld_16,
                          int32_t shadow_dtype, const uint8_t *valid, int64_t n_rows, int32_t dim,
                          int32_t dim_pad, const float *stats, const float *queries,
                          int64_t ld_q, int32_t n_queries, int32_t k, float min_similarity,
                          int64_t id_offset, int64_t *out_ids, float *out_scores,
                          int32_t capacity, void *workspace, int64_t workspace_bytes,
                          int32_t *status, void *stream);

/* sb_cosine_topk in two phases, so a pipeline of query batches can rescore
 * one batch on a second stream while the next batch is screened.
 * sb_cosine_screen runs query preparation and the tensor-core screening into
 * the workspace; sb_cosine_rescore then rescores the workspace's candidates
 * exactly and writes out_ids / out_scores.  Both take the arguments of
 * sb_cosine_topk that they use, with the same meaning, except that
 * sb_cosine_screen zeroes *status itself (on its stream, before its kernels).
 * The rescore must see the screen's writes to the workspace and to *status
 * (same stream, or an event between the two streams), and the workspace must
 * not be reused before the rescore has finished.  Screen then rescore equals one
 * sb_cosine_topk call with the same arguments.  (No reference counterpart:
 * the reference searches one query at a time.) */
SB_API int sb_cosine_screen(const void *emb16, int64_t ld_16, int32_t shadow_dtype,
                            const uint8_t *valid, int64_t n_rows, int32_t dim, int32_t dim_pad,
                            const float *stats, const float *queries, int64_t ld_q,
                            int32_t n_queries, int32_t k, float min_similarity, int32_t capacity,
                            void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);
SB_API int sb_cosine_rescore(const float *emb, int64_t ld_emb, int64_t n_rows, int32_t dim,
                             int32_t dim_pad, int32_t n_queries, int32_t k, float min_similarity,
                             int64_t id_offset, int64_t *out_ids, float *out_scores, int32_t capacity,
                             void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);

/* Merge n_lists (<= 16) per-query sorted top-k lists into one
 * [n_queries][k] by (score desc, id asc); ids < 0 are empty.  List l is
 * [n_queries][k] at ids + l * ids_list_stride (elements; >= n_queries * k)
 * and scores + l * scores_list_stride, so the lists can sit inside the
 * per-shard records of one all-gather.  Used after an all-gather of
 * per-shard sb_cosine_topk results (no reference counterpart: the reference
 * searches one process's matrix). */
SB_API int sb_topk_merge(const int64_t *ids, int64_t ids_list_stride, const float *scores,
                         int64_t scores_list_stride, int32_t n_lists, int32_t n_queries, int32_t k,
                         int64_t *out_ids, float *out_scores, void *stream);

/* ------------------------------------------------------------------------ */
/* Partial-prefill attention                                                */
/* ------------------------------------------------------------------------ */
/* A [batch, heads, seq, head_dim] tensor with a contiguous last dimension;
 * strides are in elements. */
typedef struct sb_attn_tensor {
  void *data;
  int64_t stride_batch, stride_head, stride_seq;
} sb_attn_tensor;

/* Compact a per-batch compute mask (uint8, [batch][seq_len] with batch stride
 * mask_stride) into ascending row indices rows[b*rows_stride + i] and
 * counts[b] (device int32), with no host synchronisation.  Replaces the mask
 * scan of _partial_prefill_attention_kernel
 * (semblend_core/triton_kernels.py:571-581) and the .item() of
 * partial_prefill_attention (:680). */
SB_API int sb_mask_to_rows(const uint8_t *mask, int64_t mask_stride, int32_t batch, int32_t seq_len,
                           int32_t *rows, int64_t rows_stride, int32_t *counts, void *stream);

/* Causal attention at compute rows only, with grouped-query attention:
 * for b < batch, i < counts[b], p = rows[b*rows_stride + i] (ascending) and
 * query head h, out[b,h,p] = softmax(q[b,h,p] . k[b,g,0..p]^T * scale)
 * v[b,g,0..p] with g = h / (n_q_heads / n_kv_heads); other rows of out are
 * not written.  max_rows bounds every counts[b].  bf16 / fp16 with
 * head_dim 128 run on the tensor cores (fp32 accumulation and softmax);
 * other head dims (<= 256) and fp32 run on CUDA cores.  *status (device
 * int32, zeroed by the caller) receives a value >= 2 if a kernel wait timed
 * out.  The tensor-core kernel hands out its work units from a counter pair
 * inside the library (one of 64 per device, taken round robin per call and
 * reset by the call's last CTA): at most 64 calls may be in flight on one
 * device at a time, and the first call on a device looks the counters up
 * (make it before any stream capture).
 *
 * Replaces partial_prefill_attention (semblend_core/triton_kernels.py:655-734;
 * kernel :532-652), which has the same math for n_q_heads == n_kv_heads and
 * batch 1. */
SB_API int sb_partial_attention(sb_attn_tensor q, sb_attn_tensor k, sb_attn_tensor v, sb_attn_tensor out,
                                const int32_t *rows, int64_t rows_stride, const int32_t *counts,
                                int32_t max_rows, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                int32_t seq_len, int32_t head_dim, float scale, int32_t dtype,
                                int32_t *status, void *stream);

/* ------------------------------------------------------------------------ */
/* Masked QKV projection                                                    */
/* ------------------------------------------------------------------------ */
/* Workspace bytes sb_masked_linear needs (the compacted rows of x; 0 for fp32). */
SB_API int64_t sb_masked_linear_workspace_bytes(int32_t n_rows, int32_t in_features, int32_t dtype);

/* out[rows[i], :] = x[rows[i], :] @ w^T (+ bias) for i < n_rows, with fp32
 * accumulation and one rounding to the element type; other rows of out are
 * not written (zero them first for the reference's output).  x [*, ldx],
 * w [out_features, ldw], out [*, ldo], bias [out_features] or NULL, all of
 * `dtype`; rows device int32.  bf16 / fp16 with 16-byte aligned rows
 * (in_features, ldx, ldw, ldo multiples of 8) run a tcgen05 GEMM over the
 * compacted rows only; fp32 and other 16-bit shapes run on CUDA cores.
 * *status (device int32, zeroed by the caller)
 * receives a value >= 2 if a kernel wait timed out.
 *
 * Replaces masked_qkv_projection (semblend_core/triton_kernels.py:451-522;
 * kernel :366-448), which computes every row and then zeroes the reuse rows. */
SB_API int sb_masked_linear(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *bias,
                            const int32_t *rows, int32_t n_rows, int32_t out_features,
                            int32_t in_features, void *out, int64_t ldo, int32_t dtype,
                            void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);

/* ------------------------------------------------------------------------ */
/* Chunk-hash alignment                                                     */
/* ------------------------------------------------------------------------ */
/* SHA-256 of every full chunk of `chunk` token ids (device int32 / int64,
 * SB_INDEX_*), each id packed as a little-endian uint32; the first 128 bits of
 * each digest as four big-endian words: digests[n_tokens / chunk][4].  A
 * trailing partial chunk is not hashed.  Replaces _chunk_hash
 * (semblend_core/alignment.py:120-130) over the chunks of
 * compute_chunk_alignment (:170-180) and estimate_reuse_ratio (:752-774). */
SB_API int sb_chunk_digests(const void *tokens, int32_t token_dtype, int64_t n_tokens, int32_t chunk,
                            uint32_t *digests, void *stream);

/* Exact chunk matching of compute_chunk_alignment (alignment.py:181-252):
 * full target chunk t (in order) takes the first donor chunk with its digest
 * that no earlier target chunk took; with context_gate != 0 a match survives
 * only if target chunk t - 1 or t + 1 also matched.  Writes match[t] (device
 * int32, donor chunk or -1) for the n_target_chunks full target chunks and
 * the position pairs of the matched chunks in target order,
 * donor_positions[i] / target_positions[i] (device int32, all
 * n_target_chunks * chunk entries written: -1 after the *n_pairs valid
 * ones), with their count in *n_pairs (device int64) — the inputs of
 * sb_inject, built without the host (the -1 entries are skipped there).
 * n_target_chunks <= 65536. */
SB_API int sb_chunk_align(const uint32_t *donor_digests, int32_t n_donor_chunks,
                          const uint32_t *target_digests, int32_t n_target_chunks, int32_t chunk,
                          int32_t context_gate, int32_t *match, int32_t *donor_positions,
                          int32_t *target_positions, int64_t *n_pairs, void *stream);

/* sb_chunk_align for n_requests (donor, target) pairs in two launches.
 * offsets (device int32 [3][n_requests + 1], prefix sums) give request r its
 * donor digests [offsets[r], offsets[r + 1]) of donor_digests, its full
 * target chunks [t0, t1) = [offsets[s + r], offsets[s + r + 1]) of
 * target_digests (s = n_requests + 1) with pair slots [t0 * chunk, t1 * chunk)
 * of donor_positions / target_positions, and its match entries
 * [offsets[2s + r], offsets[2s + r + 1]) of match: its full target chunks,
 * then -1 for a trailing partial chunk.  n_pairs[r] gets request r's pair
 * count (-1 if its offsets are inconsistent or it has more than
 * max_target_chunks full target chunks; nothing else is written for it).
 * max_target_chunks (<= 65536) is the largest t1 - t0.  Positions are
 * relative to each request's own sequences; each donor's chunk count times
 * chunk must fit in int32 (the caller's offsets are not range-checked beyond
 * the per-request consistency above). */
SB_API int sb_chunk_align_batch(const uint32_t *donor_digests, const uint32_t *target_digests,
                                const int32_t *offsets, int32_t n_requests, int32_t max_target_chunks,
                                int32_t chunk, int32_t context_gate, int32_t *match,
                                int32_t *donor_positions, int32_t *target_positions, int64_t *n_pairs,
                                void *stream);

/* Workspace bytes of sb_token_overlap (8-byte aligned). */
SB_API int64_t sb_token_overlap_workspace_bytes(int64_t n_donor_tokens, int64_t n_target_tokens);

/* Multiset overlap of two token sequences (device int32 / int64 ids,
 * SB_INDEX_*): *overlap (device int64) = sum over ids of min(occurrences in
 * donor, occurrences in target) — the token-count fallback of
 * estimate_reuse_ratio (semblend_core/alignment.py:776-785), where each target
 * token consumes one unused occurrence in the donor.  Ids compare as 64-bit
 * integers (an int32 id equals the int64 id of the same value).
 * n_donor_tokens + n_target_tokens < 2^31. */
SB_API int sb_token_overlap(const void *donor_tokens, int32_t donor_dtype, int64_t n_donor_tokens,
                            const void *target_tokens, int32_t target_dtype, int64_t n_target_tokens,
                            void *workspace, int64_t workspace_bytes, int64_t *overlap, void *stream);

/* ------------------------------------------------------------------------ */
/* Miscellaneous                                                            */
/* ------------------------------------------------------------------------ */
SB_API const char *sb_status_string(int status);
SB_API int sb_version(void);
/* The last CUDA error code seen by this library on the calling thread (0 if
 * none), for diagnosing SB_ERR_CUDA. */
SB_API int sb_last_cuda_error(void);

/* Timing of the dominant kernel of each later call (inject_kernel for
 * sb_inject / sb_permute_paged, the tensor-core screening kernel for
 * sb_cosine_topk, the attention kernel for sb_partial_attention, the GEMM for
 * sb_masked_linear): CUDA events are recorded on the launch stream around each
 * of the next max_launches such launches.  sb_profile_stop synchronises on
 * them, reports the summed milliseconds and the number of launches timed, and
 * turns timing off. */
SB_API int sb_profile_start(int32_t max_launches);
SB_API int sb_profile_stop(float *total_ms, int32_t *n_launches);

/* Failure-detection self-test: launches one CTA that waits on an mbarrier
 * nothing arrives on, gives up after max_cycles clock cycles and writes 7 to
 * *status (device int32, zeroed by the caller), the way every pipelined
 * kernel here reports a stalled wait instead of hanging.  No reference
 * counterpart (the reference has no device-side waits). */
SB_API int sb_selftest_wait_timeout(int32_t *status, int64_t max_cycles, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SEMBLEND_B200_H */

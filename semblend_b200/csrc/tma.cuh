// Host-side TMA tensor-map encoding through the driver entry point (so the
// library needs no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace sb {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major bf16 matrix [rows, cols] with a row pitch in bytes, loaded in
// boxes of box_cols x box_rows with the 128-byte swizzle; out-of-range rows
// read as zeros.  Returns false if the map cannot be encoded.
inline bool make_tmap_bf16_2d(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                              uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), gdim, gstride, box,
                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D row-major 16-bit matrix (bf16 or fp16, `dtype`), otherwise as
// make_tmap_bf16_2d.
inline bool make_tmap_16_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t cols,
                            uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void *>(base), gdim, gstride, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D bf16 tensor [d2, d1, cols] with pitches in bytes (dim 1 and dim 2),
// boxes of box_cols x box_rows x 1, 128-byte swizzle, zero fill out of range.
inline bool make_tmap_bf16_3d(CUtensorMap *map, const void *base, uint64_t cols, uint64_t d1, uint64_t d2,
                              uint64_t pitch1, uint64_t pitch2, uint32_t box_cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t gdim[3] = {cols, d1, d2};
  cuuint64_t gstride[2] = {pitch1, pitch2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), gdim, gstride, box,
                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace sb

namespace sb {
// 4-D tensor [d3, d2, d1, cols] (cols contiguous) with byte pitches for
// dims 1..3, boxes of box_cols x box_rows x 1 x 1, 128-byte swizzle, zero
// fill out of range.  `dtype` is a CUtensorMapDataType (bf16 or fp16).
inline bool make_tmap_4d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t cols,
                         uint64_t d1, uint64_t d2, uint64_t d3, uint64_t p1, uint64_t p2, uint64_t p3,
                         uint32_t box_cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t gdim[4] = {cols, d1, d2, d3};
  cuuint64_t gstride[3] = {p1, p2, p3};
  cuuint32_t box[4] = {box_cols, box_rows, 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype, 4, const_cast<void *>(base), gdim, gstride, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
}  // namespace sb

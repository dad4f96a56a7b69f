// Host side of the TMA (cp.async.bulk.tensor) copies: tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lw {

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (the library links the static runtime only).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 2-D tiled tensor map: `rows` rows of `cols` elements, row stride `stride`
// bytes, box {box_cols, box_rows}; reads past the edges fill zeros.
inline bool encode_2d(CUtensorMap* m, CUtensorMapDataType type, const void* ptr, uint64_t cols, uint64_t rows,
                      uint64_t stride, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return enc(m, type, 2, const_cast<void*>(ptr), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace lw

namespace lw {

// 3-D tiled tensor map over dims {d0, d1, d2} (d0 innermost, contiguous) with
// byte strides s1 (dim 1) and s2 (dim 2), box {b0, b1, b2}. The strides need
// not grow with the dimension: a row-major [rows][bytes] matrix viewed as
// {128 bytes, rows, bytes / 128} (s1 = row bytes, s2 = 128) gives boxes whose
// shared-memory image is [chunk][row][128 bytes].
inline bool encode_3d(CUtensorMap* m, CUtensorMapDataType type, const void* ptr, uint64_t d0, uint64_t d1,
                      uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                      CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t elem[3] = {1, 1, 1};
  return enc(m, type, 3, const_cast<void*>(ptr), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace lw

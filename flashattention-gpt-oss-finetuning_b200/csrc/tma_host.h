// tma_host.h -- host-side creation of TMA tensor maps through the driver entry point
// (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace swa {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

inline CUtensorMapSwizzle swizzle_for_row_bytes(int row_bytes) {
  switch (row_bytes) {
    case 32: return CU_TENSOR_MAP_SWIZZLE_32B;
    case 64: return CU_TENSOR_MAP_SWIZZLE_64B;
    default: return CU_TENSOR_MAP_SWIZZLE_128B;
  }
}

// Tensor map over a [B, H, L, D] 16-bit tensor (element strides sb, sh, sl; dim 3 stride 1).
// Box: {box_d, box_rows, box_heads, 1}; swizzle width = box_d * 2 bytes (32, 64 or 128).
// Rows past L (and any other out-of-range coordinate) read as zero.  A box of several heads
// lands in shared memory as [box_heads][box_rows][box_d].
inline bool make_tmap_bhld(CUtensorMap* m, const void* base, int B, int H, int L, int D,
                           int64_t sb, int64_t sh, int64_t sl, int box_d, int box_rows,
                           int box_heads = 1) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const int64_t e = 2;
  // A dimension of extent 1 may carry any stride; give it a legal one.
  if (H == 1) sh = sl * (L > 0 ? L : 1);
  if (B == 1) sb = sh * H;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sl * e), (cuuint64_t)(sh * e), (cuuint64_t)(sb * e)};
  cuuint32_t box[4] = {(cuuint32_t)box_d, (cuuint32_t)box_rows, (cuuint32_t)box_heads, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for_row_bytes(box_d * 2),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map over a row-major [rows, cols] 16-bit matrix (row pitch `ld` elements).
inline bool make_tmap_2d(CUtensorMap* m, const void* base, int rows, int cols, int64_t ld,
                         int box_cols, int box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for_row_bytes(box_cols * 2),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map over a row-major [rows, cols] fp32 matrix (row pitch `ld` elements, a multiple of
// 4), no swizzle, box {box_cols, box_rows}.
inline bool make_tmap_rows_f32(CUtensorMap* m, const void* base, long long rows, int cols, int64_t ld,
                               int box_cols, int box_rows = 1) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace swa

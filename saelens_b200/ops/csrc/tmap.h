// Host-side TMA descriptor construction through the driver entry point (no -lcuda needed).
#pragma once

#include <c10/util/Exception.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include "check.h"

namespace sb {

inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    SB_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D row-major tensor [rows, cols] with `row_stride_bytes` between rows; the box is
// [box_rows, box_cols] elements.  TMA needs a 16-byte aligned base and row stride.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                                uint32_t box_rows, uint32_t box_cols,
                                CUtensorMapSwizzle swizzle) {
  SB_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  SB_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  SB_CHECK((uint64_t(box_cols) * elem_bytes) % 16 == 0, "TMA box inner extent");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  SB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return m;
}

// 3-D tensor [d2][d1][d0] (d0 contiguous) with byte strides s1 (between d1 rows) and s2 (between
// d2 planes); the box is [b2][b1][b0] elements.  Out-of-range rows of a box read as zero.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                                uint64_t d1, uint64_t d2, uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0,
                                uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
  SB_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  SB_CHECK(s1_bytes % 16 == 0 && s2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  SB_CHECK((uint64_t(b0) * elem_bytes) % 16 == 0, "TMA box inner extent");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  SB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed with code ", int(r));
  return m;
}

}  // namespace sb

// Host-side TMA descriptor construction through the driver entry point (no -lcuda needed).
#pragma once

#include <c10/util/Exception.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

namespace sb {

inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
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
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK((uint64_t(box_cols) * elem_bytes) % 16 == 0, "TMA box inner extent");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return m;
}

}  // namespace sb

// Host-side TMA descriptor construction.  cuTensorMapEncodeTiled is a driver API; it is
// resolved once through the runtime's driver-entry-point query so the extension does not
// link libcuda directly (it loads on machines without a GPU driver, e.g. for CPU tests).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include "host_check.h"

#include <mutex>

namespace b200 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  B200_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  return fn;
}

// 2-D tiled map over a row-major matrix [rows, cols] with row stride `ld` (elements).
// Box = [box_rows, box_cols]; out-of-range elements read as zero.
inline CUtensorMap make_tma_2d(void* base, CUtensorMapDataType dtype, int elem_bytes,
                               uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                               uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * elem_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  B200_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  B200_REQUIRE((ld * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUresult r = get_encode_tiled()(&m, dtype, 2, base, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B200_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed");
  return m;
}

}  // namespace b200

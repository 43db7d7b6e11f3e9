// Host-side TMA tensor-map encoding through the driver entry point (no
// link-time dependency on libcuda: the module imports without a GPU).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace b200 {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

// 2-D tiled map over a row-major matrix [rows, cols] (row stride in
// elements); box = [box_rows, box_cols], box_cols the contiguous extent.
// Out-of-range elements read as zero.
inline CUtensorMap make_tma_2d(const void* base, CUtensorMapDataType dtype, size_t esz, uint64_t rows,
                               uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                               CUtensorMapSwizzle swizzle) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * esz) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if ((box_cols * esz) % 16 != 0) throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {row_stride_elems * esz};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, dtype, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return map;
}

// 3-D tiled map over a batch of row-major matrices [batch][rows, cols] (strides in elements); box =
// [1, box_rows, box_cols].
inline CUtensorMap make_tma_3d(const void* base, CUtensorMapDataType dtype, size_t esz, uint64_t rows, uint64_t cols,
                               uint64_t batch, uint64_t row_stride_elems, uint64_t batch_stride_elems,
                               uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * esz) % 16 != 0 || (batch_stride_elems * esz) % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if ((box_cols * esz) % 16 != 0) throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t gdim[3] = {cols, rows, batch};
  cuuint64_t gstride[2] = {row_stride_elems * esz, batch_stride_elems * esz};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&map, dtype, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3-D) failed: " + std::to_string((int)r));
  return map;
}

}  // namespace b200

// Host-side helpers for building TMA tensor maps (cuTensorMapEncodeTiled),
// resolved through the runtime's driver entry-point query so the extension
// needs no direct link against libcuda.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace raiccl {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// Row-major 2-D tensor [rows, cols] with a [box_rows, box_cols] box and the
// 128-byte swizzle (box_cols * elem_bytes must equal 128).
inline CUtensorMap make_tmap_2d_sw128(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                      uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                                      uint32_t box_rows, uint32_t box_cols) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((row_stride_elems * elem_bytes) % 16 != 0)
    throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if (box_cols * elem_bytes != 128)
    throw std::runtime_error("SW128 box must be 128 bytes wide");
  if (box_rows > 256) throw std::runtime_error("TMA box rows must be <= 256");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (cuuint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return map;
}

}  // namespace raiccl

// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the extension does not link libcuda).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace b200 {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2D row-major tensor [rows, cols] with a row stride in bytes; box [box_rows, box_cols].
// cols is the innermost (contiguous) dimension.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                                uint32_t box_rows, uint32_t box_cols,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B,
                                CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  CUtensorMap m;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if ((uint64_t)box_cols * elem_bytes % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 3D tensor [d2, d1, d0] (d0 innermost) with explicit byte strides for d1 and d2.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t d2, uint64_t d1, uint64_t d0, uint64_t stride1_bytes,
                                uint64_t stride2_bytes, uint32_t box2, uint32_t box1,
                                uint32_t box0,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if ((uint64_t)box0 * elem_bytes % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tmap_encode_fn()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled(3d) failed: " + std::to_string((int)r));
  return m;
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (!cached[device]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cached[device] = v > 0 ? v : 148;
  }
  return cached[device];
}

}  // namespace b200

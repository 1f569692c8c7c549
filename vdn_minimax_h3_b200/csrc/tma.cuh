// Host-side TMA descriptor construction (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so nothing links libcuda directly).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

namespace vdn {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

// The encode call is a driver API call: it needs a current context on the calling thread.
// A thread whose first CUDA work is a tensor-map encode (autograd's backward threads, where
// PyTorch skips cudaSetDevice when the device already matches) has none and the encode
// fails with CUDA_ERROR_INVALID_CONTEXT; binding the device's primary context once per
// thread and device fixes that.
inline void bind_current_context() {
  thread_local int bound = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (bound != dev) {
    cudaSetDevice(dev);
    bound = dev;
  }
}

inline EncodeTiledFn encode_tiled_fn() {
  bind_current_context();
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Row-major 2D tensor [outer, inner] with `row_stride_bytes` between rows; box
// [box_outer, box_inner] elements; 128-byte swizzle (box_inner * elem == 128).
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                                uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if ((box_inner * elem_bytes) % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 3D tensor [d2, d1, d0] (d0 innermost) with byte strides s1 (between d1 rows) and s2.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                                uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (s1_bytes % 16 != 0 || s2_bytes % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed: " + std::to_string((int)r));
  return m;
}

inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

}  // namespace vdn

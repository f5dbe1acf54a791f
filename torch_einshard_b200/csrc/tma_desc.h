// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the extension needs no direct libcuda link).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace es {

// L2 promotion of TMA loads (0 none, 1 64B, 2 128B, 3 256B); 256B by default.
inline int& tma_l2_promotion() {
  static int mode = 3;
  return mode;
}
inline CUtensorMapL2promotion l2_promotion() {
  switch (tma_l2_promotion()) {
    case 0: return CU_TENSOR_MAP_L2_PROMOTION_NONE;
    case 1: return CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
    case 2: return CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
    default: return CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("einshard: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D tiled map over a strided tensor.  dims/strides are innermost-first;
// strides are in elements for dims 1 and 2 (dim 0 is contiguous).  128-byte
// swizzle, zero fill outside the tensor.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                                uint64_t d1, uint64_t d2, uint64_t s1_elems, uint64_t s2_elems, uint32_t box0,
                                uint32_t box1, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_elems * elem_bytes, s2_elems * elem_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  auto encode = [&]() {
    return encode_tiled_fn()(&map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2_promotion(),
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    // Threads that never touched the runtime (e.g. the autograd engine's worker)
    // have no current driver context; bind the device's primary context and retry.
    int dev = 0;
    cudaGetDevice(&dev);
    cudaSetDevice(dev);
    cudaFree(nullptr);
    r = encode();
  }
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("einshard: cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return map;
}

// N-D tiled map (rank 1..5).  dims/box innermost-first; strides in bytes for
// dims 1..rank-1.  128-byte swizzle, zero fill outside the tensor.
inline CUtensorMap make_tmap_nd(const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                                const uint64_t* strides_bytes, const uint32_t* box,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap map;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  auto encode = [&]() {
    return encode_tiled_fn()(&map, dtype, rank, const_cast<void*>(base), d, st, bx, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2_promotion(),
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaSetDevice(dev);
    cudaFree(nullptr);
    r = encode();
  }
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("einshard: cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return map;
}

}  // namespace es

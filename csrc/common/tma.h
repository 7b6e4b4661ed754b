// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the extension needs no direct libcuda link).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmt {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// cuTensorMapEncodeTiled is a driver call and needs a current context on the calling thread.
// A thread that has made no runtime call yet (PyTorch's autograd worker, when a backward
// starts with one of our ops) has none: a no-op runtime call binds the device's primary
// context, then the encode is retried.
template <typename F>
inline CUresult encode_with_context(F&& encode) {
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    cudaFree(nullptr);
    r = encode();
  }
  return r;
}

// Result of the last cuTensorMapEncodeTiled call on this thread (for error messages).
inline int& last_tmap_result() {
  static thread_local int r = 0;
  return r;
}

// True when a 2D bf16/fp32 operand can be described by a TMA map (checked before encoding).
inline bool tma_ok(const void* ptr, uint64_t ld, int elem_bytes) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * elem_bytes) % 16 == 0;
}

// Row-major 2D matrix of `outer` rows x `inner` elements (row pitch `ld` elements),
// tiled in boxes of box_outer rows x box_inner elements with 128-byte swizzling.
// Returns false if the driver rejects the description.
inline bool make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  auto fn = tmap_encode_fn();
  last_tmap_result() = fn ? -2 : -1;
  if (!fn || !tma_ok(ptr, ld, elem_bytes)) return false;
  CUresult r = encode_with_context([&] {
    return fn(m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  });
  last_tmap_result() = (int)r;
  return r == CUDA_SUCCESS;
}

// 3D map: dims (inner, mid, outer) with pitches (ld_mid, ld_outer) in elements.
inline bool make_tmap_3d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                         uint64_t mid, uint64_t outer, uint64_t ld_mid, uint64_t ld_outer, uint32_t box_inner,
                         uint32_t box_mid, uint32_t box_outer, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {ld_mid * (uint64_t)elem_bytes, ld_outer * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {box_inner, box_mid, box_outer};
  cuuint32_t estr[3] = {1, 1, 1};
  auto fn = tmap_encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || strides[0] % 16 || strides[1] % 16) return false;
  CUresult r = encode_with_context([&] {
    return fn(m, dtype, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  });
  return r == CUDA_SUCCESS;
}

}  // namespace llmt

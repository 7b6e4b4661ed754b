// Shared helpers for every llmt CUDA kernel (sm_100a only).
//
// Vector load/store wrappers, bf16 conversion, warp reductions and the launch-check
// macro used by all translation units of the extension.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <torch/extension.h>

#define LLMT_CHECK(cond, ...) TORCH_CHECK(cond, "llmt: ", __VA_ARGS__)
#define LLMT_CHECK_CUDA(t) LLMT_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define LLMT_CHECK_CONTIG(t) LLMT_CHECK((t).is_contiguous(), #t " must be contiguous")
#define LLMT_CHECK_DTYPE(t, dt) LLMT_CHECK((t).scalar_type() == (dt), #t " has dtype ", (t).scalar_type(), ", expected ", (dt))
#define LLMT_LAUNCH_CHECK() C10_CUDA_KERNEL_LAUNCH_CHECK()

namespace llmt {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline int sm_count() {
  static int n = -1;
  if (n < 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte vector of 8 bf16 values.
struct alignas(16) BF16x8 {
  bf162 h[4];
};

__device__ __forceinline__ void bf16x8_to_float(const BF16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ BF16x8 float_to_bf16x8(const float* f) {
  BF16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float4 ld_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st_f4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  bf162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace llmt

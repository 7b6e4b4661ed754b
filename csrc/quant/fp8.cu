// Tensorwise e4m3 quantization for the fp8 linears.
//
// Same recipe as the reference's _fp8_quant_impl / _fp8_quant_t_impl (kernels/lowp.py:51-62):
// amax = max |x| over the whole tensor (at least 1e-12), scale = 448 / amax (as 448 * (1 / amax)),
// q = e4m3(clamp(x * scale, -448, 448)) rounded to nearest even, and the inverse scale
// 1 / scale that the GEMM multiplies back in. The reference runs this as torch.compile'd
// Triton; here it is two kernels with no atomics and no memset, so it captures in a CUDA graph:
//   pass 1  a fixed grid of kAmaxBlocks CTAs writes one partial max each into scratch
//   pass 2  every CTA reduces those partials itself (a few hundred floats from L2), quantizes a
//           64 x 64 tile with 16-byte loads and stores, and, when asked, writes the transposed
//           tile (through shared memory) into qt, the copy the backward GEMMs read K-major.
#include <cuda_fp8.h>

#include "../common/common.cuh"

namespace llmt {
namespace {

constexpr int kAmaxBlocks = 296;  // two per SM
constexpr int kQThreads = 256;
constexpr int kTile = 64;
constexpr int kPitch = kTile + 4;  // transposed-tile row pitch in bytes (2-way bank conflicts at most)

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* v);
template <>
__device__ __forceinline__ void load16<bf16>(const bf16* p, float* v) {
  bf16x8_to_float(*reinterpret_cast<const BF16x8*>(p), v);
  bf16x8_to_float(*reinterpret_cast<const BF16x8*>(p + 8), v + 8);
}
template <>
__device__ __forceinline__ void load16<float>(const float* p, float* v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = ld_f4(p + 4 * i);
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

__device__ __forceinline__ float block_max(float m, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = m;
  __syncthreads();
  m = l < kQThreads / 32 ? red[l] : 0.f;
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return __shfl_sync(0xffffffffu, m, 0);
}

template <typename T>
__global__ void __launch_bounds__(kQThreads) fp8_amax_kernel(const T* __restrict__ x, int rows, int cols, int64_t ld,
                                                             float* __restrict__ partial) {
  pdl_wait();
  __shared__ float red[kQThreads / 32];
  const int gpr = cols / 16;  // 16-element groups per row
  const int64_t n = (int64_t)rows * gpr;
  const int64_t stride = (int64_t)gridDim.x * kQThreads;
  float m = 0.f;
  if (ld == cols) {  // contiguous: no row / column split (a 64-bit division per group costs more than the load)
    for (int64_t i = (int64_t)blockIdx.x * kQThreads + threadIdx.x; i < n; i += stride) {
      float v[16];
      load16(x + i * 16, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
    }
  } else {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {  // a row per CTA, its groups over the threads
      for (int i = threadIdx.x; i < gpr; i += kQThreads) {
        float v[16];
        load16(x + (int64_t)r * ld + i * 16, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
      }
    }
  }
  m = block_max(m, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = m;
  pdl_trigger();
}

template <typename T>
__global__ void __launch_bounds__(kQThreads) fp8_quant_kernel(const T* __restrict__ x, int rows, int cols, int64_t ld,
                                                              const float* __restrict__ partial, uint8_t* __restrict__ q,
                                                              uint8_t* __restrict__ qt, float* __restrict__ inv) {
  pdl_wait();
  __shared__ float red[kQThreads / 32];
  __shared__ __align__(16) uint8_t tile[kTile * kPitch];  // [col][row] of the quantized tile
  float m = 0.f;
  for (int i = threadIdx.x; i < kAmaxBlocks; i += kQThreads) m = fmaxf(m, partial[i]);
  const float amax = fmaxf(block_max(m, red), 1e-12f);
  // the reference evaluates 448 / amax as reciprocal(amax) * 448 (PyTorch's scalar / tensor)
  const float scale = __fmul_rn(__frcp_rn(amax), 448.f);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *inv = __frcp_rn(scale);

  const int r0 = blockIdx.y * kTile, c0 = blockIdx.x * kTile;
  const int tr = threadIdx.x >> 2, tc = (threadIdx.x & 3) * 16;
  const int r = r0 + tr, c = c0 + tc;
  if (r < rows && c < cols) {
    float v[16];
    load16(x + (int64_t)r * ld + c, v);
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // satfinite clamps to +-448, the same as the reference's clamp before the cast
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(v[4 * e] * scale, v[4 * e + 1] * scale), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(v[4 * e + 2] * scale, v[4 * e + 3] * scale), __NV_SATFINITE, __NV_E4M3);
      w[e] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(q + (int64_t)r * cols + c) = make_uint4(w[0], w[1], w[2], w[3]);
    if (qt) {
#pragma unroll
      for (int e = 0; e < 16; ++e) tile[(tc + e) * kPitch + tr] = (uint8_t)(w[e >> 2] >> (8 * (e & 3)));
    }
  }
  if (qt) {
    __syncthreads();
    // qt row c0 + j holds x's column c0 + j: 64 rows' bytes, 16 per thread
    const int j = threadIdx.x >> 2, k = (threadIdx.x & 3) * 16;
    if (c0 + j < cols && r0 + k < rows) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(tile + j * kPitch + k);
      *reinterpret_cast<uint4*>(qt + (int64_t)(c0 + j) * rows + r0 + k) = make_uint4(src[0], src[1], src[2], src[3]);
    }
  }
  pdl_trigger();
}

template <typename T>
void launch_quant(const T* x, int rows, int cols, int64_t ld, uint8_t* q, uint8_t* qt, float* inv, float* scratch,
                  cudaStream_t st) {
  launch_pdl(fp8_amax_kernel<T>, kAmaxBlocks, kQThreads, 0, st, x, rows, cols, ld, scratch);
  dim3 grid((unsigned)cdiv(cols, kTile), (unsigned)cdiv(rows, kTile));
  launch_pdl(fp8_quant_kernel<T>, grid, kQThreads, 0, st, x, rows, cols, ld, (const float*)scratch, q, qt, inv);
}

}  // namespace

int fp8_amax_slots() { return kAmaxBlocks; }

cudaError_t fp8_quant(const void* x, bool x_f32, int rows, int cols, int64_t ld, void* q, void* qt, float* inv,
                      float* scratch, cudaStream_t st) {
  LLMT_REQUIRE(rows % 16 == 0 && cols % 16 == 0, "fp8_quant: rows and cols must be multiples of 16");
  LLMT_REQUIRE(ld % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0, "fp8_quant: x needs 16-byte alignment");
  LLMT_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(qt) & 15) == 0,
               "fp8_quant: outputs need 16-byte alignment");
  if (rows == 0 || cols == 0) return cudaSuccess;
  if (x_f32)
    launch_quant(static_cast<const float*>(x), rows, cols, ld, static_cast<uint8_t*>(q), static_cast<uint8_t*>(qt), inv,
                 scratch, st);
  else
    launch_quant(static_cast<const bf16*>(x), rows, cols, ld, static_cast<uint8_t*>(q), static_cast<uint8_t*>(qt), inv,
                 scratch, st);
  return cudaGetLastError();
}

}  // namespace llmt

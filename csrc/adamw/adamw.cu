// Fused AdamW over one flat parameter buffer (sm_100a).
//
// Same update as torch.optim.AdamW used by the reference (bench_train.py:467-469,
// lr 3e-4, betas (0.9, 0.95), wd 0.1, eps 1e-8), decoupled weight decay:
//   p *= 1 - lr*wd;  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// and in the same pass writes the bf16 shadow copy that the GEMMs read, so no separate
// weight cast kernel runs per step (the autocast casts of the reference, roofline.py:164).
// The step count t and lr live on the device so a captured CUDA graph replays correctly.
// grad_scale multiplies g first (DP averaging / loss scaling folded in). With zero_grad the
// kernel also clears g after reading it, so every gradient producer of the next step can
// accumulate (TMA reduce-add, split-K) without a separate zeroing pass.
#include "../common/common.cuh"

namespace llmt {
namespace {

template <bool WRITE_BF16, bool ZERO_GRAD>
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p16, int64_t n, const float* __restrict__ lr_ptr,
                             const int* __restrict__ step_ptr, AdamHyper a) {
  pdl_wait();
  const float lr = *lr_ptr;
  const int t = *step_ptr;
  const float bc1 = 1.f - powf(a.b1, (float)t);
  const float bc2 = 1.f - powf(a.b2, (float)t);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * a.wd;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = ld_f4(p + 4 * i), gg = ld_f4(g + 4 * i), mm = ld_f4(m + 4 * i), vv = ld_f4(v + 4 * i);
    float* pe = &pp.x;
    float* ge = &gg.x;
    float* me = &mm.x;
    float* ve = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = ge[j] * a.grad_scale;
      me[j] = a.b1 * me[j] + (1.f - a.b1) * gj;
      ve[j] = a.b2 * ve[j] + (1.f - a.b2) * gj * gj;
      const float denom = sqrtf(ve[j]) * inv_sqrt_bc2 + a.eps;
      pe[j] = pe[j] * decay - step_size * me[j] / denom;
    }
    st_f4(p + 4 * i, pp);
    if (ZERO_GRAD) st_f4(g + 4 * i, make_float4(0.f, 0.f, 0.f, 0.f));
    st_f4(m + 4 * i, mm);
    st_f4(v + 4 * i, vv);
    if (WRITE_BF16) {
      uint2 o;
      o.x = pack_bf16x2(pp.x, pp.y);
      o.y = pack_bf16x2(pp.z, pp.w);
      *reinterpret_cast<uint2*>(p16 + 4 * i) = o;
    }
  }
  // tail (n not a multiple of 4)
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const int64_t i = n4 * 4 + threadIdx.x;
    const float gj = g[i] * a.grad_scale;
    const float mj = a.b1 * m[i] + (1.f - a.b1) * gj;
    const float vj = a.b2 * v[i] + (1.f - a.b2) * gj * gj;
    const float pj = p[i] * decay - step_size * mj / (sqrtf(vj) * inv_sqrt_bc2 + a.eps);
    m[i] = mj;
    v[i] = vj;
    p[i] = pj;
    if (ZERO_GRAD) g[i] = 0.f;
    if (WRITE_BF16) p16[i] = __float2bfloat16_rn(pj);
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ x, bf16* __restrict__ y, int64_t n) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

// 8 elements per thread and iteration (two 16-byte loads, one 16-byte store), two iterations'
// loads issued before either store: enough bytes in flight per SM for a grid of a few SMs (the
// overlapped data-parallel step casts on the SMs the backward leaves free).
__global__ void cast_bf16_x8_kernel(const float* __restrict__ x, bf16* __restrict__ y, int64_t n8) {
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += 2 * stride) {
    const int64_t j = i + stride;
    const float4 a0 = ld_f4(x + 8 * i), a1 = ld_f4(x + 8 * i + 4);
    float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
    if (j < n8) {
      b0 = ld_f4(x + 8 * j);
      b1 = ld_f4(x + 8 * j + 4);
    }
    *reinterpret_cast<uint4*>(y + 8 * i) = make_uint4(pack_bf16x2(a0.x, a0.y), pack_bf16x2(a0.z, a0.w),
                                                      pack_bf16x2(a1.x, a1.y), pack_bf16x2(a1.z, a1.w));
    if (j < n8)
      *reinterpret_cast<uint4*>(y + 8 * j) = make_uint4(pack_bf16x2(b0.x, b0.y), pack_bf16x2(b0.z, b0.w),
                                                        pack_bf16x2(b1.x, b1.y), pack_bf16x2(b1.z, b1.w));
  }
}

}  // namespace

// zero_grad: also reset g to 0 after reading it (the next step's gradients accumulate into it).
// max_blocks > 0 caps the grid (a side stream sharing the GPU with the backward).
cudaError_t adamw_step(float* p, float* g, float* m, float* v, void* p16, int64_t n, const float* lr,
                       const int* step, AdamHyper h, bool zero_grad, cudaStream_t st, int max_blocks) {
  if (n == 0) return cudaSuccess;
  LLMT_REQUIRE(((uintptr_t)p | (uintptr_t)g | (uintptr_t)m | (uintptr_t)v) % 16 == 0,
               "adamw: fp32 buffers must be 16-byte aligned");
  LLMT_REQUIRE(p16 == nullptr || (uintptr_t)p16 % 8 == 0, "adamw: bf16 copy must be 8-byte aligned");
  const int64_t cap = max_blocks > 0 ? max_blocks : sm_count() * 8;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n / 4 + 1, 256), cap));
  bf16* q = static_cast<bf16*>(p16);
  if (p16 && zero_grad) launch_pdl(adamw_kernel<true, true>, grid, 256, 0, st, p, g, m, v, q, n, lr, step, h);
  else if (p16) launch_pdl(adamw_kernel<true, false>, grid, 256, 0, st, p, g, m, v, q, n, lr, step, h);
  else if (zero_grad) launch_pdl(adamw_kernel<false, true>, grid, 256, 0, st, p, g, m, v, nullptr, n, lr, step, h);
  else launch_pdl(adamw_kernel<false, false>, grid, 256, 0, st, p, g, m, v, nullptr, n, lr, step, h);
  return cudaGetLastError();
}

// max_blocks > 0 caps the grid (a side stream that must leave the rest of the GPU to others).
cudaError_t cast_bf16(const float* x, void* y, int64_t n, cudaStream_t st, int max_blocks) {
  if (n == 0) return cudaSuccess;
  const int64_t cap = max_blocks > 0 ? max_blocks : sm_count() * 8;
  if (n % 8 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 16) == 0) {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n / 8, 512), cap));
    launch_pdl(cast_bf16_x8_kernel, grid, 256, 0, st, x, static_cast<bf16*>(y), n / 8);
  } else {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), cap));
    launch_pdl(cast_bf16_kernel, grid, 256, 0, st, x, static_cast<bf16*>(y), n);
  }
  return cudaGetLastError();
}

}  // namespace llmt

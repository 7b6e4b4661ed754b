// Fused AdamW over one flat parameter buffer (sm_100a).
//
// Same update as torch.optim.AdamW used by the reference (bench_train.py:467-469,
// lr 3e-4, betas (0.9, 0.95), wd 0.1, eps 1e-8), decoupled weight decay:
//   p *= 1 - lr*wd;  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// and in the same pass writes the bf16 shadow copy that the GEMMs read, so no separate
// weight cast kernel runs per step (the autocast casts of the reference, roofline.py:164).
// The step count t and lr live on the device so a captured CUDA graph replays correctly.
// grad_scale multiplies g first (DP averaging / loss scaling folded in).
#include "../common/common.cuh"

namespace llmt {
namespace {

struct AdamArgs {
  float b1, b2, eps, wd, grad_scale;
};

template <bool WRITE_BF16>
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p16, int64_t n, const float* __restrict__ lr_ptr,
                             const int* __restrict__ step_ptr, AdamArgs a) {
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
    if (WRITE_BF16) p16[i] = __float2bfloat16_rn(pj);
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ x, bf16* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

}  // namespace

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p16,
                at::Tensor lr, at::Tensor step, double b1, double b2, double eps, double wd, double grad_scale) {
  for (auto* t : {&p, &g, &m, &v}) {
    LLMT_CHECK_DTYPE((*t), at::kFloat);
    LLMT_CHECK_CONTIG((*t));
  }
  LLMT_CHECK(g.numel() == p.numel() && m.numel() == p.numel() && v.numel() == p.numel(), "adamw: size mismatch");
  LLMT_CHECK_DTYPE(lr, at::kFloat);
  LLMT_CHECK_DTYPE(step, at::kInt);
  const bool w16 = p16.has_value() && p16->defined();
  if (w16) {
    LLMT_CHECK_DTYPE((*p16), at::kBFloat16);
    LLMT_CHECK(p16->numel() == p.numel(), "adamw: bf16 copy size mismatch");
  }
  const int64_t n = p.numel();
  if (n == 0) return;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n / 4 + 1, 256), sm_count() * 8));
  AdamArgs a{(float)b1, (float)b2, (float)eps, (float)wd, (float)grad_scale};
  auto kern = w16 ? adamw_kernel<true> : adamw_kernel<false>;
  kern<<<grid, 256, 0, cur_stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                       v.data_ptr<float>(), w16 ? reinterpret_cast<bf16*>(p16->data_ptr()) : nullptr, n,
                                       lr.data_ptr<float>(), step.data_ptr<int>(), a);
  LLMT_LAUNCH_CHECK();
}

void cast_bf16(at::Tensor x, at::Tensor y) {
  LLMT_CHECK_DTYPE(x, at::kFloat);
  LLMT_CHECK_DTYPE(y, at::kBFloat16);
  LLMT_CHECK(x.numel() == y.numel() && x.is_contiguous() && y.is_contiguous(), "cast_bf16: bad args");
  const int64_t n = x.numel();
  if (n == 0) return;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), sm_count() * 8));
  cast_bf16_kernel<<<grid, 256, 0, cur_stream()>>>(x.data_ptr<float>(), reinterpret_cast<bf16*>(y.data_ptr()), n);
  LLMT_LAUNCH_CHECK();
}

}  // namespace llmt

// Memory-bound elementwise kernels: SwiGLU fwd/bwd, RoPE fwd/bwd on the packed qkv
// layout, embedding gather / scatter-add.
//
// SwiGLU (reference kernels/triton_ops.py:172-194): h = silu(g) * u,
//   dg = dh * u * sig(g) * (1 + g * (1 - sig(g))),  du = dh * silu(g).
// g and u are read through a row stride so the same kernel serves the merged w1||w3
// GEMM output (N, 2*ffn) = [g | u] and two separate (N, ffn) tensors. The native training
// path fuses both directions into GEMM epilogues; these are the standalone ops.
//
// RoPE (reference bench_train.py:83-100, triton_ops.py:226-287): rotate-half on the q and
// k heads of the packed qkv rows (N, (H + 2*KV) * hd), in place; v is untouched. The
// attention kernels read q, k, v straight from this packed layout, so no (3,B,H,T,hd)
// copy exists. Backward applies the transposed rotation in place on the packed dqkv.
//   y1 = x1 c - x2 s, y2 = x2 c + x1 s;   dx1 = dy1 c + dy2 s, dx2 = dy2 c - dy1 s
// with c, s from the (T, hd) fp32 tables (halves duplicated, reference layout).
#include "../common/common.cuh"

namespace llmt {
namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void swiglu_fwd_kernel(const bf16* __restrict__ g, const bf16* __restrict__ u, int64_t ldgu,
                                  bf16* __restrict__ h, int64_t ldh, int64_t rows, int F) {
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    float gf[8], uf[8], o[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(g + r * ldgu + c), gf);
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(u + r * ldgu + c), uf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = gf[j] * sigmoidf_(gf[j]) * uf[j];
    *reinterpret_cast<BF16x8*>(h + r * ldh + c) = float_to_bf16x8(o);
  }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dh, int64_t lddh, const bf16* __restrict__ g,
                                  const bf16* __restrict__ u, int64_t ldgu, bf16* __restrict__ dg,
                                  bf16* __restrict__ du, int64_t lddgu, int64_t rows, int F) {
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    float gf[8], uf[8], d[8], og[8], ou[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(g + r * ldgu + c), gf);
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(u + r * ldgu + c), uf);
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(dh + r * lddh + c), d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = sigmoidf_(gf[j]);
      og[j] = d[j] * uf[j] * sg * (1.f + gf[j] * (1.f - sg));
      ou[j] = d[j] * gf[j] * sg;
    }
    *reinterpret_cast<BF16x8*>(dg + r * lddgu + c) = float_to_bf16x8(og);
    *reinterpret_cast<BF16x8*>(du + r * lddgu + c) = float_to_bf16x8(ou);
  }
}

// One thread per (token, rotated head, 8-wide chunk of the first half).
template <bool BWD>
__global__ void rope_kernel(bf16* __restrict__ qkv, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int64_t N, int T, int n_rot_heads, int hd, int64_t ld) {
  const int half = hd / 2;
  const int chunks = half / 8;
  const int64_t total = N * n_rot_heads * chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % chunks) * 8;
    const int64_t rest = i / chunks;
    const int h = (int)(rest % n_rot_heads);
    const int64_t n = rest / n_rot_heads;
    const int t = (int)(n % T);
    bf16* base = qkv + n * ld + (int64_t)h * hd;
    float x1[8], x2[8], y1[8], y2[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(base + c), x1);
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(base + half + c), x2);
    const float* cr = cos_t + (int64_t)t * hd;
    const float* sr = sin_t + (int64_t)t * hd;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float c1 = cr[c + j], s1 = sr[c + j], c2 = cr[half + c + j], s2 = sr[half + c + j];
      if (!BWD) {
        y1[j] = x1[j] * c1 - x2[j] * s1;
        y2[j] = x2[j] * c2 + x1[j] * s2;
      } else {
        y1[j] = x1[j] * c1 + x2[j] * s2;
        y2[j] = x2[j] * c2 - x1[j] * s1;
      }
    }
    *reinterpret_cast<BF16x8*>(base + c) = float_to_bf16x8(y1);
    *reinterpret_cast<BF16x8*>(base + half + c) = float_to_bf16x8(y2);
  }
}

__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ W,
                                     float* __restrict__ x, int64_t N, int d, int64_t V, int* __restrict__ err) {
  const int vpr = d / 4;
  const int64_t total = N * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / vpr;
    const int c = (int)(i % vpr) * 4;
    int64_t tok = idx[n];
    if (tok < 0 || tok >= V) {  // record and clamp instead of reading out of bounds
      if (err) atomicExch(err, 1);
      tok = 0;
    }
    st_f4(x + n * d + c, ld_f4(W + tok * d + c));
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ dx,
                                     float* __restrict__ dW, int64_t N, int d, int64_t V) {
  const int vpr = d / 4;
  const int64_t total = N * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / vpr;
    const int c = (int)(i % vpr) * 4;
    const int64_t tok = idx[n];
    if (tok < 0 || tok >= V) continue;
    atomicAdd(reinterpret_cast<float4*>(dW + tok * d + c), ld_f4(dx + n * d + c));
  }
}

inline int ew_grid(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)sm_count() * 16));
}

}  // namespace

void swiglu_fwd(at::Tensor g, at::Tensor u, at::Tensor h) {
  LLMT_CHECK_DTYPE(g, at::kBFloat16);
  LLMT_CHECK_DTYPE(u, at::kBFloat16);
  LLMT_CHECK_DTYPE(h, at::kBFloat16);
  LLMT_CHECK(g.dim() == 2 && u.dim() == 2 && h.dim() == 2, "SwiGLU operands must be 2D");
  const int F = g.size(1);
  const int64_t rows = g.size(0);
  LLMT_CHECK(F % 8 == 0, "SwiGLU width must be a multiple of 8");
  LLMT_CHECK(g.stride(1) == 1 && u.stride(1) == 1 && h.stride(1) == 1, "SwiGLU inner dim must be contiguous");
  LLMT_CHECK(g.stride(0) == u.stride(0), "g and u must share a row stride");
  if (rows == 0) return;
  swiglu_fwd_kernel<<<ew_grid(rows * F / 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(g.data_ptr()), reinterpret_cast<const bf16*>(u.data_ptr()), g.stride(0),
      reinterpret_cast<bf16*>(h.data_ptr()), h.stride(0), rows, F);
  LLMT_LAUNCH_CHECK();
}

void swiglu_bwd(at::Tensor dh, at::Tensor g, at::Tensor u, at::Tensor dg, at::Tensor du) {
  LLMT_CHECK(g.dim() == 2 && u.dim() == 2 && dh.dim() == 2 && dg.dim() == 2 && du.dim() == 2,
             "SwiGLU operands must be 2D");
  const int F = g.size(1);
  const int64_t rows = g.size(0);
  LLMT_CHECK(F % 8 == 0, "SwiGLU width must be a multiple of 8");
  LLMT_CHECK(g.stride(0) == u.stride(0) && dg.stride(0) == du.stride(0), "paired row strides differ");
  if (rows == 0) return;
  swiglu_bwd_kernel<<<ew_grid(rows * F / 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(dh.data_ptr()), dh.stride(0), reinterpret_cast<const bf16*>(g.data_ptr()),
      reinterpret_cast<const bf16*>(u.data_ptr()), g.stride(0), reinterpret_cast<bf16*>(dg.data_ptr()),
      reinterpret_cast<bf16*>(du.data_ptr()), dg.stride(0), rows, F);
  LLMT_LAUNCH_CHECK();
}

// qkv: (B*T, (H + 2*KV) * hd) bf16, rotated in place. n_rot_heads = H + KV (q and k heads).
void rope_inplace(at::Tensor qkv, at::Tensor cos_t, at::Tensor sin_t, int64_t T, int64_t n_rot_heads, int64_t hd,
                  bool backward) {
  LLMT_CHECK_DTYPE(qkv, at::kBFloat16);
  LLMT_CHECK_DTYPE(cos_t, at::kFloat);
  LLMT_CHECK(hd % 16 == 0, "head dim must be a multiple of 16");
  LLMT_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous(), "rope tables must be contiguous");
  LLMT_CHECK(cos_t.size(0) >= T && cos_t.size(1) == hd, "rope table too small");
  LLMT_CHECK(qkv.is_contiguous(), "qkv must be contiguous");
  const int64_t ld = qkv.size(-1);
  const int64_t N = qkv.numel() / ld;
  const int64_t work = N * n_rot_heads * (hd / 16);
  if (work == 0) return;
  auto kern = backward ? rope_kernel<true> : rope_kernel<false>;
  kern<<<ew_grid(work), 256, 0, cur_stream()>>>(reinterpret_cast<bf16*>(qkv.data_ptr()), cos_t.data_ptr<float>(),
                                                 sin_t.data_ptr<float>(), N, (int)T, (int)n_rot_heads, (int)hd, ld);
  LLMT_LAUNCH_CHECK();
}

void embedding_fwd(at::Tensor idx, at::Tensor W, at::Tensor x, c10::optional<at::Tensor> err) {
  LLMT_CHECK_DTYPE(idx, at::kLong);
  LLMT_CHECK_DTYPE(W, at::kFloat);
  LLMT_CHECK(W.size(1) % 4 == 0, "embedding width must be a multiple of 4");
  LLMT_CHECK(idx.is_contiguous() && W.is_contiguous() && x.is_contiguous(), "embedding operands must be contiguous");
  const int64_t N = idx.numel();
  const int d = W.size(1);
  if (N == 0) return;
  embedding_fwd_kernel<<<ew_grid(N * d / 4), 256, 0, cur_stream()>>>(
      idx.data_ptr<int64_t>(), W.data_ptr<float>(), x.data_ptr<float>(), N, d, W.size(0),
      (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr);
  LLMT_LAUNCH_CHECK();
}

// dW += scatter(dx by idx). The caller zeroes dW for the first micro-batch.
void embedding_bwd(at::Tensor idx, at::Tensor dx, at::Tensor dW) {
  LLMT_CHECK_DTYPE(dx, at::kFloat);
  LLMT_CHECK_DTYPE(dW, at::kFloat);
  LLMT_CHECK(dx.is_contiguous() && dW.is_contiguous(), "embedding grads must be contiguous");
  const int64_t N = idx.numel();
  const int d = dW.size(1);
  if (N == 0) return;
  embedding_bwd_kernel<<<ew_grid(N * d / 4), 256, 0, cur_stream()>>>(idx.data_ptr<int64_t>(), dx.data_ptr<float>(),
                                                                      dW.data_ptr<float>(), N, d, dW.size(0));
  LLMT_LAUNCH_CHECK();
}

}  // namespace llmt

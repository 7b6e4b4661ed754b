// Cross entropy over rows of a materialized logits chunk (sm_100a).
//
// The chunked lm-head + cross-entropy of the reference (kernels/triton_ops.py:330-405)
// writes a chunk of logits and runs a per-row kernel over it. The native training path
// never writes logits (the CE reductions run in the lm-head GEMM epilogue, csrc/gemm);
// these row kernels remain as the standalone op for callers that already hold logits.
//   forward  lse = log sum exp(row), loss = lse - row[target]
//   backward row := (softmax(row) - onehot(target)) * grad_out * scale, in place
// Online max/sum-exp per thread, then a block reduction (Milakov & Gimelshein 2018).
// One 256-thread CTA per row; 16-byte vector loads.
#include "../common/common.cuh"

namespace llmt {
namespace {

constexpr int kCeThreads = 256;

__device__ __forceinline__ void online_combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

__device__ __forceinline__ void block_lse(float& m, float& s) {
  __shared__ float sm[kCeThreads / 32], ss[kCeThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_combine(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  m = sm[0];
  s = ss[0];
  for (int i = 1; i < kCeThreads / 32; ++i) online_combine(m, s, sm[i], ss[i]);
}

__global__ void __launch_bounds__(kCeThreads)
ce_fwd_rows_kernel(const bf16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ tgt, float* __restrict__ lse,
                   float* __restrict__ loss, int V) {
  pdl_wait();
  const int64_t r = blockIdx.x;
  const bf16* row = logits + r * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
    if (!LLMT_IN(r * ld + c, r * ld + c + 8, (int64_t)(gridDim.x - 1) * ld + V, 301)) continue;
    float f[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(row + c), f);
    float mx = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mx = fmaxf(mx, f[j]);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += __expf(f[j] - mx);
    online_combine(m, s, mx, sum);
  }
  block_lse(m, s);
  if (threadIdx.x == 0) {
    const float l = m + logf(s);
    lse[r] = l;
    const int64_t t = tgt[r];
    loss[r] = (t >= 0 && t < V) ? l - __bfloat162float(row[t]) : 0.f;
  }
}

__global__ void __launch_bounds__(kCeThreads)
ce_bwd_rows_kernel(bf16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ tgt, const float* __restrict__ lse,
                   const float* __restrict__ grad_out, float scale, int V) {
  pdl_wait();
  const int64_t r = blockIdx.x;
  bf16* row = logits + r * ld;
  const float l = lse[r];
  const float g = scale * (grad_out ? *grad_out : 1.f);
  const int64_t t = tgt[r];
  for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
    if (!LLMT_IN(r * ld + c, r * ld + c + 8, (int64_t)(gridDim.x - 1) * ld + V, 302)) continue;
    float f[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(row + c), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (__expf(f[j] - l) - ((c + j) == t ? 1.f : 0.f)) * g;
    *reinterpret_cast<BF16x8*>(row + c) = float_to_bf16x8(f);
  }
}

}  // namespace

cudaError_t ce_fwd_rows(const void* logits, int64_t ld, const int64_t* tgt, float* lse, float* loss, int64_t R, int V,
                        cudaStream_t st) {
  LLMT_REQUIRE(V % 8 == 0 && ld % 8 == 0, "ce: vocab and pitch must be multiples of 8");
  if (R == 0) return cudaSuccess;
  launch_pdl(ce_fwd_rows_kernel, (unsigned)R, kCeThreads, 0, st, static_cast<const bf16*>(logits), ld, tgt, lse, loss, V);
  return cudaGetLastError();
}

cudaError_t ce_bwd_rows(void* logits, int64_t ld, const int64_t* tgt, const float* lse, const float* grad_out,
                        float scale, int64_t R, int V, cudaStream_t st) {
  LLMT_REQUIRE(V % 8 == 0 && ld % 8 == 0, "ce: vocab and pitch must be multiples of 8");
  if (R == 0) return cudaSuccess;
  launch_pdl(ce_bwd_rows_kernel, (unsigned)R, kCeThreads, 0, st, static_cast<bf16*>(logits), ld, tgt, lse, grad_out, scale, V);
  return cudaGetLastError();
}

}  // namespace llmt

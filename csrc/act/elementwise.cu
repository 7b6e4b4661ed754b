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
  pdl_wait();
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    // the last row ends F columns after its start: extents of the strided g / u / h views
    if (!LLMT_IN(r * ldgu + c, r * ldgu + c + 8, (rows - 1) * ldgu + F, 201) ||
        !LLMT_IN(r * ldh + c, r * ldh + c + 8, (rows - 1) * ldh + F, 202))
      continue;
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
  pdl_wait();
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    if (!LLMT_IN(r * ldgu + c, r * ldgu + c + 8, (rows - 1) * ldgu + F, 203) ||
        !LLMT_IN(r * lddh + c, r * lddh + c + 8, (rows - 1) * lddh + F, 204) ||
        !LLMT_IN(r * lddgu + c, r * lddgu + c + 8, (rows - 1) * lddgu + F, 205))
      continue;
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
  pdl_wait();
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
    // the rotated heads of the last row end n_rot_heads * hd columns after its start; the
    // tables hold T rows of hd
    if (!LLMT_IN(n * ld + (int64_t)h * hd + c, n * ld + (int64_t)h * hd + half + c + 8,
                 (N - 1) * ld + (int64_t)n_rot_heads * hd, 210) ||
        !LLMT_IN((int64_t)t * hd + c, (int64_t)t * hd + half + c + 8, (int64_t)T * hd, 211))
      continue;
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

// W holds vocabulary rows [v0, v0 + V). With `partial` (a vocabulary-parallel shard) ids
// outside that range give zero rows; otherwise they are an error (recorded, row 0 used).
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ W,
                                     float* __restrict__ x, int64_t N, int d, int64_t V, int64_t v0, bool partial,
                                     int* __restrict__ err) {
  pdl_wait();
  const int vpr = d / 4;
  const int64_t total = N * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / vpr;
    const int c = (int)(i % vpr) * 4;
    int64_t tok = idx[n] - v0;
    if (tok < 0 || tok >= V) {
      if (partial) {
        st_f4(x + n * d + c, make_float4(0.f, 0.f, 0.f, 0.f));
        continue;
      }
      if (err) atomicExch(err, 1);  // record and clamp instead of reading out of bounds
      tok = 0;
    }
    if (!LLMT_IN(tok * d + c, tok * d + c + 4, V * d, 220) || !LLMT_IN(n * d + c, n * d + c + 4, N * d, 221)) continue;
    st_f4(x + n * d + c, ld_f4(W + tok * d + c));
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ dx,
                                     float* __restrict__ dW, int64_t N, int d, int64_t V, int64_t v0) {
  pdl_wait();
  const int vpr = d / 4;
  const int64_t total = N * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / vpr;
    const int c = (int)(i % vpr) * 4;
    const int64_t tok = idx[n] - v0;
    if (tok < 0 || tok >= V) continue;
    if (!LLMT_IN(tok * d + c, tok * d + c + 4, V * d, 222) || !LLMT_IN(n * d + c, n * d + c + 4, N * d, 223)) continue;
    atomicAdd(reinterpret_cast<float4*>(dW + tok * d + c), ld_f4(dx + n * d + c));
  }
}

inline int ew_grid(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)sm_count() * 16));
}

}  // namespace

cudaError_t swiglu_fwd(const void* g, const void* u, int64_t ldgu, void* h, int64_t ldh, int64_t rows, int F,
                       cudaStream_t st) {
  LLMT_REQUIRE(F % 8 == 0 && ldgu % 8 == 0 && ldh % 8 == 0, "swiglu: widths and pitches must be multiples of 8");
  if (rows == 0) return cudaSuccess;
  launch_pdl(swiglu_fwd_kernel, ew_grid(rows * F / 8), 256, 0, st, static_cast<const bf16*>(g), static_cast<const bf16*>(u),
                                                           ldgu, static_cast<bf16*>(h), ldh, rows, F);
  return cudaGetLastError();
}

cudaError_t swiglu_bwd(const void* dh, int64_t lddh, const void* g, const void* u, int64_t ldgu, void* dg, void* du,
                       int64_t lddgu, int64_t rows, int F, cudaStream_t st) {
  LLMT_REQUIRE(F % 8 == 0 && ldgu % 8 == 0 && lddh % 8 == 0 && lddgu % 8 == 0,
               "swiglu: widths and pitches must be multiples of 8");
  if (rows == 0) return cudaSuccess;
  launch_pdl(swiglu_bwd_kernel, ew_grid(rows * F / 8), 256, 0, st, static_cast<const bf16*>(dh), lddh,
                                                           static_cast<const bf16*>(g), static_cast<const bf16*>(u),
                                                           ldgu, static_cast<bf16*>(dg), static_cast<bf16*>(du), lddgu,
                                                           rows, F);
  return cudaGetLastError();
}

// qkv: (N, ld) bf16 rows; the first n_rot_heads heads (q and k) are rotated in place.
cudaError_t rope_inplace(void* qkv, const float* cos_t, const float* sin_t, int64_t N, int T, int n_rot_heads, int hd,
                         int64_t ld, bool backward, cudaStream_t st) {
  LLMT_REQUIRE(hd % 16 == 0 && ld % 8 == 0, "rope: head dim must be a multiple of 16");
  const int64_t work = N * n_rot_heads * (hd / 16);
  if (work == 0) return cudaSuccess;
  auto kern = backward ? rope_kernel<true> : rope_kernel<false>;
  launch_pdl(kern, ew_grid(work), 256, 0, st, static_cast<bf16*>(qkv), cos_t, sin_t, N, T, n_rot_heads, hd, ld);
  return cudaGetLastError();
}

cudaError_t embedding_fwd(const int64_t* idx, const float* W, float* x, int64_t N, int d, int64_t V, int64_t v0,
                          bool partial, int* err, cudaStream_t st) {
  LLMT_REQUIRE(d % 4 == 0, "embedding: width must be a multiple of 4");
  if (N == 0) return cudaSuccess;
  launch_pdl(embedding_fwd_kernel, ew_grid(N * d / 4), 256, 0, st, idx, W, x, N, d, V, v0, partial, err);
  return cudaGetLastError();
}

// dW += scatter(dx by idx - v0); ids outside [v0, v0 + V) are skipped. The caller zeroes dW
// for the first micro-batch.
cudaError_t embedding_bwd(const int64_t* idx, const float* dx, float* dW, int64_t N, int d, int64_t V, int64_t v0,
                          cudaStream_t st) {
  LLMT_REQUIRE(d % 4 == 0, "embedding: width must be a multiple of 4");
  if (N == 0) return cudaSuccess;
  launch_pdl(embedding_bwd_kernel, ew_grid(N * d / 4), 256, 0, st, idx, dx, dW, N, d, V, v0);
  return cudaGetLastError();
}

}  // namespace llmt

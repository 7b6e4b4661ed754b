#include <stdlib.h>

#include <atomic>
// Fused residual-add + RMSNorm, forward and backward (sm_100a).
//
// Contract (same math as the reference's add+RMSNorm, kernels/cuda_ext/add_rmsnorm.cu:78-178
// and kernels/triton_ops.py:38-86):
//   forward   s = r + a (a optional), rstd = 1/sqrt(mean(s^2) + eps), y = s * rstd * w
//   backward  g = dy * w, c = mean(g * s), ds = rstd * g - s * rstd^3 * c + ds_in,
//             dw = sum_rows dy * s * rstd
// Dtypes on the native path: a bf16 (a GEMM output), r/s fp32 (the residual stream),
// w fp32 (master weight), y bf16 (the next GEMM's operand), ds fp32 + a bf16 copy.
//
// Layout: TPR threads per row (a power of two, 32..256), each owning up to 4 chunks of 8
// consecutive elements, 256 threads per CTA (256/TPR rows per CTA). The backward is
// persistent; every CTA keeps its dw partial in registers and writes one (D) partial row,
// and a column-parallel reduce kernel sums the partials in a fixed order (deterministic dw;
// the reference reduces its (P, D) partials with a separate dwp.sum(0), add_rmsnorm_ext.py:70).
#include "../common/common.cuh"

namespace llmt {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 4;

template <int TPR>
__device__ __forceinline__ float row_sum(float v, float* red) {
  v = warp_sum(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    constexpr int WPR = TPR / 32;  // warps per row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_in_cta = threadIdx.x / TPR;
    __syncthreads();  // protect red[] from the previous use
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < WPR; ++i) t += red[row_in_cta * WPR + i];
    return t;
  }
}

template <int TPR, bool HAS_A, bool WRITE_S>
__global__ void __launch_bounds__(kThreads)
add_rmsnorm_fwd_kernel(const bf16* __restrict__ a, const float* __restrict__ r, const float* __restrict__ w,
                       bf16* __restrict__ y, float* __restrict__ s_out, float* __restrict__ rstd_out,
                       int64_t N, int D, float eps) {
  pdl_wait();
  __shared__ float red[kThreads / 32];
  constexpr int RPC = kThreads / TPR;
  const int t = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * RPC + threadIdx.x / TPR;
  const bool valid = row < N;
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int e = (c * TPR + t) * 8;
    if (valid && e < D && LLMT_IN(row * D + e, row * D + e + 8, N * D, 101)) {
      const int64_t off = row * D + e;
      float4 r0 = ld_f4(r + off), r1 = ld_f4(r + off + 4);
      v[c][0] = r0.x; v[c][1] = r0.y; v[c][2] = r0.z; v[c][3] = r0.w;
      v[c][4] = r1.x; v[c][5] = r1.y; v[c][6] = r1.z; v[c][7] = r1.w;
      if constexpr (HAS_A) {
        float af[8];
        bf16x8_to_float(*reinterpret_cast<const BF16x8*>(a + off), af);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] += af[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
    }
  }
  ss = row_sum<TPR>(ss, red);
  const float rstd = rsqrtf(ss / (float)D + eps);
  if (!valid) return;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int e = (c * TPR + t) * 8;
    if (e < D && LLMT_IN(row * D + e, row * D + e + 8, N * D, 102) && LLMT_IN(e, e + 8, D, 103)) {
      const int64_t off = row * D + e;
      if constexpr (WRITE_S) {
        st_f4(s_out + off, make_float4(v[c][0], v[c][1], v[c][2], v[c][3]));
        st_f4(s_out + off + 4, make_float4(v[c][4], v[c][5], v[c][6], v[c][7]));
      }
      float4 w0 = ld_f4(w + e), w1 = ld_f4(w + e + 4);
      float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * rstd * ww[j];
      *reinterpret_cast<BF16x8*>(y + off) = float_to_bf16x8(o);
    }
  }
  if (t == 0 && LLMT_IN(row, row + 1, N, 104)) rstd_out[row] = rstd;
}

// dy bf16, s fp32, ds_in fp32 (optional); ds fp32 and ds16 bf16 (optional) out.
// Two passes over each row's registers-free chunks (the second re-reads dy and s from L1).
// The dw partial of a row group lives in its own shared-memory row (each thread owns its 8-column
// pieces, so no synchronisation), not in registers: the kernel then fits five CTAs per SM and
// one wave covers the 4096 rows of a medium step (a second, mostly idle wave cost a whole
// dependent DRAM round trip). Each CTA writes one (D) dw partial row; dw_reduce_kernel sums
// them in a fixed order.
template <int TPR, bool HAS_DSIN, bool WRITE_DS16>
__global__ void __launch_bounds__(kThreads)
rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const float* __restrict__ s, const float* __restrict__ w,
                   const float* __restrict__ rstd_in, const float* __restrict__ ds_in,
                   float* __restrict__ ds, bf16* __restrict__ ds16, float* __restrict__ dw_part, int64_t N, int D) {
  pdl_wait();
  __shared__ float red[kThreads / 32];
  extern __shared__ float sdw[];  // [RPC][D] dw partials, one row per row group
  constexpr int RPC = kThreads / TPR;
  const int t = threadIdx.x % TPR;
  const int rgroup = threadIdx.x / TPR;
  float* my_dw = sdw + (int64_t)rgroup * D;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int e = (c * TPR + t) * 8;
    if (e < D) {
      reinterpret_cast<float4*>(my_dw + e)[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(my_dw + e)[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const int64_t stride = (int64_t)gridDim.x * RPC;
  // Every row group runs the same number of iterations so the block-wide barriers in
  // row_sum line up; rows past N are masked.
  const int64_t iters = cdiv(N, stride);
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t row = it * stride + (int64_t)blockIdx.x * RPC + rgroup;
    const bool valid = row < N;
    float dot = 0.f;
    const float rs = (valid && LLMT_IN(row, row + 1, N, 110)) ? rstd_in[row] : 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int e = (c * TPR + t) * 8;
      if (valid && e < D && LLMT_IN(row * D + e, row * D + e + 8, N * D, 111) && LLMT_IN(e, e + 8, D, 112)) {
        const int64_t off = row * D + e;
        if constexpr (HAS_DSIN) {
          // the second pass adds ds_in after the row reduction: start its DRAM fetch now so that
          // pass finds it in L2 instead of paying a second dependent DRAM round trip
          asm volatile("prefetch.global.L2 [%0];" ::"l"(ds_in + off));
        }
        float dyf[8];
        bf16x8_to_float(*reinterpret_cast<const BF16x8*>(dy + off), dyf);
        const float4 s0 = ld_f4(s + off), s1 = ld_f4(s + off + 4);
        const float4 w0 = ld_f4(w + e), w1 = ld_f4(w + e + 4);
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float4* acc = reinterpret_cast<float4*>(my_dw + e);
        float4 a0 = acc[0], a1 = acc[1];
        float* av0 = reinterpret_cast<float*>(&a0);
        float* av1 = reinterpret_cast<float*>(&a1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dot += dyf[j] * wv[j] * sv[j];
          (j < 4 ? av0[j] : av1[j - 4]) += dyf[j] * sv[j] * rs;
        }
        acc[0] = a0;
        acc[1] = a1;
      }
    }
    dot = row_sum<TPR>(dot, red);
    const float cc = dot / (float)D;
    const float rs3 = rs * rs * rs;
    if (valid) {
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int e = (c * TPR + t) * 8;
        if (e < D && LLMT_IN(row * D + e, row * D + e + 8, N * D, 113) && LLMT_IN(e, e + 8, D, 114)) {
          const int64_t off = row * D + e;
          float dyf[8];
          bf16x8_to_float(*reinterpret_cast<const BF16x8*>(dy + off), dyf);
          const float4 s0 = ld_f4(s + off), s1 = ld_f4(s + off + 4);
          const float4 w0 = ld_f4(w + e), w1 = ld_f4(w + e + 4);
          const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
          const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = rs * dyf[j] * wv[j] - sv[j] * rs3 * cc;
          if constexpr (HAS_DSIN) {
            const float4 d0 = ld_f4(ds_in + off), d1 = ld_f4(ds_in + off + 4);
            o[0] += d0.x; o[1] += d0.y; o[2] += d0.z; o[3] += d0.w;
            o[4] += d1.x; o[5] += d1.y; o[6] += d1.z; o[7] += d1.w;
          }
          st_f4(ds + off, make_float4(o[0], o[1], o[2], o[3]));
          st_f4(ds + off + 4, make_float4(o[4], o[5], o[6], o[7]));
          if constexpr (WRITE_DS16) *reinterpret_cast<BF16x8*>(ds16 + off) = float_to_bf16x8(o);
        }
      }
    }
  }
  // CTA-level reduction of dw over the row groups' shared-memory rows: one barrier, then each
  // thread sums whole columns over the row groups in a fixed order.
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += kThreads) {
    float a = 0.f;
#pragma unroll
    for (int rg = 0; rg < RPC; ++rg) a += sdw[rg * D + i];
    if (LLMT_IN((int64_t)blockIdx.x * D + i, (int64_t)blockIdx.x * D + i + 1, (int64_t)gridDim.x * D, 115))
      dw_part[(int64_t)blockIdx.x * D + i] = a;
  }
  pdl_trigger();
}

// dw[j] (+)= sum_p part[p, j] in a fixed order (deterministic): 4 columns x 64 row groups per CTA,
// each thread summing every 64th partial (a few independent L2 loads), then a fixed shared-memory
// tree over the 64 groups. D / 4 CTAs keep the whole GPU busy on the ~1 MB of partials.
constexpr int kRedCols = 4, kRedGroups = 64;
__global__ void __launch_bounds__(kRedCols * kRedGroups)
dw_reduce_kernel(const float* __restrict__ part, float* __restrict__ dw, int P, int D, int accumulate) {
  pdl_wait();
  __shared__ float acc[kRedGroups][kRedCols + 1];
  const int col = blockIdx.x * kRedCols + threadIdx.x;
  float a = 0.f;
  if (col < D)
    for (int p = threadIdx.y; p < P; p += kRedGroups)
      if (LLMT_IN((int64_t)p * D + col, (int64_t)p * D + col + 1, (int64_t)P * D, 120)) a += part[(int64_t)p * D + col];
  acc[threadIdx.y][threadIdx.x] = a;
  __syncthreads();
#pragma unroll
  for (int h = kRedGroups / 2; h > 0; h >>= 1) {
    if (threadIdx.y < h) acc[threadIdx.y][threadIdx.x] += acc[threadIdx.y + h][threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.y == 0 && col < D && LLMT_IN(col, col + 1, D, 121)) dw[col] = accumulate ? dw[col] + acc[0][threadIdx.x] : acc[0][threadIdx.x];
  pdl_trigger();
}

template <typename F>
bool dispatch_tpr(int D, F&& f) {
  if (D % 8 != 0) return false;
  if (D <= 32 * 8 * kMaxChunks) f(std::integral_constant<int, 32>{});
  else if (D <= 64 * 8 * kMaxChunks) f(std::integral_constant<int, 64>{});
  else if (D <= 128 * 8 * kMaxChunks) f(std::integral_constant<int, 128>{});
  else if (D <= 256 * 8 * kMaxChunks) f(std::integral_constant<int, 256>{});
  else return false;
  return true;
}

}  // namespace

// y = rmsnorm(r + a) * w; a (bf16) and s (fp32 out) optional.
cudaError_t add_rmsnorm_fwd(const void* a_bf16, const float* r, const float* w, void* y_bf16, float* s, float* rstd,
                            int64_t N, int D, float eps, cudaStream_t st) {
  LLMT_REQUIRE(D % 8 == 0 && D <= 8192, "rmsnorm: width must be a multiple of 8 and at most 8192");
  if (N == 0) return cudaSuccess;
  const bf16* ap = static_cast<const bf16*>(a_bf16);
  bf16* y = static_cast<bf16*>(y_bf16);
  dispatch_tpr(D, [&](auto tpr) {
    constexpr int TPR = decltype(tpr)::value;
    constexpr int RPC = kThreads / TPR;
    dim3 grid((unsigned)cdiv(N, RPC));
    auto launch = [&](auto kern) { launch_pdl(kern, grid, kThreads, 0, st, ap, r, w, y, s, rstd, N, D, eps); };
    if (ap && s) launch(add_rmsnorm_fwd_kernel<TPR, true, true>);
    else if (ap) launch(add_rmsnorm_fwd_kernel<TPR, true, false>);
    else if (s) launch(add_rmsnorm_fwd_kernel<TPR, false, true>);
    else launch(add_rmsnorm_fwd_kernel<TPR, false, false>);
  });
  return cudaGetLastError();
}

int rmsnorm_bwd_partials(int64_t N, int D) {
  int tpr = D <= 1024 ? 32 : D <= 2048 ? 64 : D <= 4096 ? 128 : 256;
  const int rpc = kThreads / tpr;
  // CTAs per SM: what the registers and the [rows per CTA][D] dw slots allow for the largest
  // variant (ds_in and the bf16 copy), so that as many rows as possible are in flight in one wave;
  // LLMT_NORM_BWD_CTAS_PER_SM overrides it for tuning
  static int env = [] {
    const char* e = getenv("LLMT_NORM_BWD_CTAS_PER_SM");
    return e ? atoi(e) : 0;
  }();
  static std::atomic<int> cached[4] = {0, 0, 0, 0};  // per threads-per-row choice (D sets the slot size)
  const int slot = tpr == 32 ? 0 : tpr == 64 ? 1 : tpr == 128 ? 2 : 3;
  int per_sm = env > 0 ? env : cached[slot].load();
  if (per_sm <= 0) {
    per_sm = 1;
    dispatch_tpr(D, [&](auto t) {
      constexpr int TPR = decltype(t)::value;
      int n = 0;
      // the slot size at this TPR's largest width, so that the answer holds for every D it serves
      const size_t smem = (size_t)(kThreads / TPR) * (TPR * 8 * kMaxChunks) * sizeof(float);
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rmsnorm_bwd_kernel<TPR, true, true>, kThreads, smem) ==
              cudaSuccess &&
          n > 0)
        per_sm = n;
      else
        (void)cudaGetLastError();
    });
    cached[slot].store(per_sm);
  }
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(N, rpc), (int64_t)per_sm * sm_count()));
}

// ds = rmsnorm backward + ds_in (optional); ds16 (bf16 copy) optional; dw written or accumulated.
// dw_part must hold rmsnorm_bwd_partials(N, D) x D floats. `ticket` is unused (kept for ABI).
cudaError_t rmsnorm_bwd(const void* dy_bf16, const float* s, const float* w, const float* rstd, const float* ds_in,
                        float* ds, void* ds16, float* dw_part, float* dw, unsigned* ticket, int64_t N, int D,
                        int accumulate, cudaStream_t st) {
  (void)ticket;
  LLMT_REQUIRE(D % 8 == 0 && D <= 8192, "rmsnorm: width must be a multiple of 8 and at most 8192");
  if (N == 0) return cudaSuccess;
  const bf16* dy = static_cast<const bf16*>(dy_bf16);
  bf16* d16 = static_cast<bf16*>(ds16);
  const int grid = rmsnorm_bwd_partials(N, D);
  dispatch_tpr(D, [&](auto tpr) {
    constexpr int TPR = decltype(tpr)::value;
    // one partial row per row group: (256 / TPR) x D floats <= 32 KB, as TPR grows with D
    const size_t smem = (size_t)(kThreads / TPR) * D * sizeof(float);
    auto launch = [&](auto kern) {
      launch_pdl(kern, grid, kThreads, smem, st, dy, s, w, rstd, ds_in, ds, d16, dw_part, N, D);
    };
    if (ds_in && d16) launch(rmsnorm_bwd_kernel<TPR, true, true>);
    else if (ds_in) launch(rmsnorm_bwd_kernel<TPR, true, false>);
    else if (d16) launch(rmsnorm_bwd_kernel<TPR, false, true>);
    else launch(rmsnorm_bwd_kernel<TPR, false, false>);
  });
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  launch_pdl(dw_reduce_kernel, (unsigned)cdiv(D, kRedCols), dim3(kRedCols, kRedGroups), 0, st, dw_part, dw, grid, D, accumulate);
  return cudaGetLastError();
}

}  // namespace llmt

// ---------------------------------------------------------------- allocation-free entry point
// See norm/noalloc.h. The dw partial sums live in this fixed device array instead of a
// buffer the caller allocates; every GPU that loads the library holds it until exit.
#include "noalloc.h"

namespace {
static __device__ __align__(256) float g_rmsnorm_noalloc_scratch[LLMT_NOALLOC_SCRATCH_FLOATS];

// Device address of the scratch array for the current device, looked up once per device
// (host code cannot use the array's name as a device pointer). The per-device slots are
// atomics, so first calls from several host threads at once are safe; they all store the
// same address. A lookup cannot run inside a stream capture (it may load the module), so a
// first call made while the stream is capturing is refused with a message.
float* noalloc_scratch_ptr(cudaStream_t stream, cudaError_t* err) {
  static std::atomic<float*> ptrs[64];
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  float* cached = ptrs[dev].load(std::memory_order_relaxed);
  if (cached) return cached;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
    llmt::set_last_error("llmt_rmsnorm_bwd_noalloc: the first call on a device must come before any stream "
                         "capture (it looks up the scratch array's device address)");
    *err = cudaErrorStreamCaptureUnsupported;
    return nullptr;
  }
  void* p = nullptr;
  *err = cudaGetSymbolAddress(&p, g_rmsnorm_noalloc_scratch);
  if (*err != cudaSuccess) return nullptr;
  ptrs[dev].store(static_cast<float*>(p), std::memory_order_relaxed);
  return static_cast<float*>(p);
}
}  // namespace

extern "C" int llmt_rmsnorm_bwd_noalloc(const void* dy_bf16, const float* s, const float* w, const float* rstd,
                                        const float* ds_in, float* ds, void* ds16, float* dw, int64_t N, int D,
                                        int accumulate, cudaStream_t stream) {
  using namespace llmt;
  if (D <= 0 || D % 8 != 0 || D > LLMT_NOALLOC_MAX_WIDTH) {
    set_last_error("llmt_rmsnorm_bwd_noalloc: width must be a positive multiple of 8 and at most 8192");
    return (int)cudaErrorInvalidValue;
  }
  if (N < 0) {
    set_last_error("llmt_rmsnorm_bwd_noalloc: negative row count");
    return (int)cudaErrorInvalidValue;
  }
  if (N == 0) return (int)cudaSuccess;
  cudaError_t e = cudaSuccess;
  float* part = noalloc_scratch_ptr(stream, &e);
  if (!part) return (int)e;
  // One partial row per CTA; the scratch holds LLMT_NOALLOC_SCRATCH_FLOATS / D of them.
  const int grid = std::max(1, std::min(rmsnorm_bwd_partials(N, D), LLMT_NOALLOC_SCRATCH_FLOATS / D));
  const bf16* dy = static_cast<const bf16*>(dy_bf16);
  bf16* d16 = static_cast<bf16*>(ds16);
  dispatch_tpr(D, [&](auto tpr) {
    constexpr int TPR = decltype(tpr)::value;
    const size_t smem = (size_t)(kThreads / TPR) * D * sizeof(float);
    auto launch = [&](auto kern) {
      launch_pdl(kern, grid, kThreads, smem, stream, dy, s, w, rstd, ds_in, ds, d16, part, N, D);
    };
    if (ds_in && d16) launch(rmsnorm_bwd_kernel<TPR, true, true>);
    else if (ds_in) launch(rmsnorm_bwd_kernel<TPR, true, false>);
    else if (d16) launch(rmsnorm_bwd_kernel<TPR, false, true>);
    else launch(rmsnorm_bwd_kernel<TPR, false, false>);
  });
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  launch_pdl(dw_reduce_kernel, (unsigned)cdiv(D, kRedCols), dim3(kRedCols, kRedGroups), 0, stream, part, dw, grid, D, accumulate);
  return (int)cudaGetLastError();
}

extern "C" const char* llmt_noalloc_last_error() { return llmt::last_error(); }

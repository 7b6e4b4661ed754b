// Data-parallel step on NVLink SHARP (NVLS) multicast, sm_100a: the gradient reduce-scatter,
// the ZeRO-1 AdamW update of this rank's shard and the all-gather of the new bf16 weights in
// one kernel, with the reductions done inside the NVSwitch.
//
// The reference only models this step (perf_model/scaling.py:163-170: a ring all-reduce of fp32
// gradients and a ZeRO-1 optimizer). Here the flat bf16 gradient buffer and the flat bf16 weight
// (shadow) buffer are symmetric allocations bound to NVLink multicast objects (set up by
// PyTorch's symmetric-memory rendezvous). For its shard [lo, lo + n) a rank
//   g = multimem.ld_reduce.add (fp32 accumulation) of the gradient at the multicast address:
//       the switch reads every rank's value and returns the sum, so each gradient byte leaves
//       its GPU once and the reduce-scatter costs no SM work beyond issuing the loads;
//   AdamW on its fp32 master / m / v shard (local memory, the math of adamw.cu);
//   multimem.st of the new bf16 weights to the multicast address: the switch writes them into
//       every rank's weight buffer (the all-gather), on the opposite link direction from the
//       reduction traffic, so the two overlap inside the one kernel.
// The gradient is cast from the fp32 buffer the backward writes to bf16 first (the bucket
// cast: half the NVLink bytes of an fp32 reduction). Ordering across ranks uses the flag
// barrier of dp_fused.cu (bounded spins with an error code) before the kernel (every rank's
// cast is complete) and after it (every rank's weights are written).
// No TMA is used here, and no multicast TMA anywhere.
#include "../common/common.cuh"

namespace llmt {
namespace {

struct NvlsArgs {
  const uint8_t* g_mc;  // multicast address of the flat bf16 gradient buffer
  uint8_t* w_mc;        // multicast address of the flat bf16 weight buffer
  float* master;        // local flat fp32 master weights (full size; the shard is updated)
  float* m;             // shard-sized Adam state
  float* v;
  int64_t lo, n;        // shard [lo, lo + n), multiples of 8
  const float* lr;
  const int* step;
  AdamHyper h;
};

__device__ __forceinline__ void mc_ld_reduce_bf16x8(const uint8_t* p, uint32_t (&r)[4]) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(p)
               : "memory");
}
__device__ __forceinline__ void mc_st_bf16x8(uint8_t* p, const uint32_t (&r)[4]) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

constexpr int kUnroll = 4;  // reductions in flight per thread (each crosses the switch)

__global__ void __launch_bounds__(256) dp_nvls_adamw_kernel(NvlsArgs a) {
  const float lr = *a.lr;
  const int t = *a.step;
  const float bc1 = 1.f - powf(a.h.b1, (float)t);
  const float bc2 = 1.f - powf(a.h.b2, (float)t);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * a.h.wd;
  const int64_t n8 = a.n / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n8; i0 += stride * kUnroll) {
    uint32_t gr[kUnroll][4];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n8) mc_ld_reduce_bf16x8(a.g_mc + (a.lo + 8 * i) * 2, gr[u]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n8) break;
      const int64_t gi = a.lo + 8 * i;
      float g[8], p[8], mm[8], vv[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const bf162*>(&gr[u][k]));
        g[2 * k] = f.x;
        g[2 * k + 1] = f.y;
      }
      *reinterpret_cast<float4*>(p) = ld_f4(a.master + gi);
      *reinterpret_cast<float4*>(p + 4) = ld_f4(a.master + gi + 4);
      *reinterpret_cast<float4*>(mm) = ld_f4(a.m + 8 * i);
      *reinterpret_cast<float4*>(mm + 4) = ld_f4(a.m + 8 * i + 4);
      *reinterpret_cast<float4*>(vv) = ld_f4(a.v + 8 * i);
      *reinterpret_cast<float4*>(vv + 4) = ld_f4(a.v + 8 * i + 4);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gk = g[k] * a.h.grad_scale;
        mm[k] = a.h.b1 * mm[k] + (1.f - a.h.b1) * gk;
        vv[k] = a.h.b2 * vv[k] + (1.f - a.h.b2) * gk * gk;
        p[k] = p[k] * decay - step_size * mm[k] / (sqrtf(vv[k]) * inv_sqrt_bc2 + a.h.eps);
      }
      st_f4(a.master + gi, *reinterpret_cast<float4*>(p));
      st_f4(a.master + gi + 4, *reinterpret_cast<float4*>(p + 4));
      st_f4(a.m + 8 * i, *reinterpret_cast<float4*>(mm));
      st_f4(a.m + 8 * i + 4, *reinterpret_cast<float4*>(mm + 4));
      st_f4(a.v + 8 * i, *reinterpret_cast<float4*>(vv));
      st_f4(a.v + 8 * i + 4, *reinterpret_cast<float4*>(vv + 4));
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = pack_bf16x2(p[2 * k], p[2 * k + 1]);
      mc_st_bf16x8(a.w_mc + gi * 2, w);
    }
  }
  __threadfence_system();
}

}  // namespace

cudaError_t dp_nvls_adamw(const void* g_mc, void* w_mc, float* master, float* m, float* v, int64_t lo, int64_t n,
                          const float* lr, const int* step, AdamHyper h, cudaStream_t st, int max_blocks) {
  LLMT_REQUIRE(n % 8 == 0 && lo % 8 == 0, "dp_nvls_adamw: shard bounds must be multiples of 8");
  LLMT_REQUIRE((reinterpret_cast<uintptr_t>(g_mc) & 15) == 0 && (reinterpret_cast<uintptr_t>(w_mc) & 15) == 0,
               "dp_nvls_adamw: multicast addresses must be 16-byte aligned");
  if (n == 0) return cudaSuccess;
  NvlsArgs a{static_cast<const uint8_t*>(g_mc), static_cast<uint8_t*>(w_mc), master, m, v, lo, n, lr, step, h};
  const int64_t cap = max_blocks > 0 ? max_blocks : sm_count() * 4;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n / 8, 256 * kUnroll), cap));
  dp_nvls_adamw_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace llmt

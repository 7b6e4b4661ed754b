// Fused data-parallel step over NVLink peer memory (sm_100a): reduce-scatter of the fp32
// gradient + ZeRO-1 AdamW on this rank's shard + all-gather of the new bf16 weights, in one
// kernel, with no NCCL call and no intermediate buffer.
//
// The reference only models this step (perf_model/scaling.py:163-170: ring all-reduce of fp32
// gradients, ZeRO-1 optimizer). Here every rank's flat gradient and bf16 shadow-weight
// buffers are CUDA-IPC mapped into every other rank (plain P2P loads/stores through NVSwitch,
// no multicast). For its shard [lo, lo + n) rank r:
//   g   = sum_p grad_p[lo + i]                 (P2P loads, 16 B per access)
//   grad_p[lo + i] = 0 for every p             (the reader clears when the next step accumulates;
//                                               skipped when its first write stores)
//   AdamW on master[lo + i], m[i], v[i]        (local, same math as adamw.cu)
//   shadow_p[lo + i] = bf16(master[lo + i])    (P2P stores: the parameter all-gather)
// Ordering across ranks uses a flag barrier before (all gradients complete) and after (all
// shards written) the update: each rank bumps a local epoch, stores it into every peer's
// signal pad with release semantics and spins, bounded by %globaltimer, on its own pad until
// every peer's slot reaches the epoch. A timeout records an error code the host can read and
// the kernel returns instead of hanging.
#include <string.h>

#include "../common/common.cuh"
#include "../common/sm100.cuh"

namespace llmt {
namespace {

constexpr uint64_t kBarrierLimitNs = 5000000000ull;  // 5 s

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: bump the epoch, publish it to every rank's pad slot [rank], wait for all slots.
__global__ void dp_barrier_kernel(uint32_t* const* pads, uint32_t* my_pad, uint32_t* epoch, int rank, int world,
                                  int* err, int code) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint32_t e = epoch[0] + 1;
  epoch[0] = e;
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(pads[p] + rank, e);
  const uint64_t t0 = sm100::globaltimer();
  for (int p = 0; p < world; ++p) {
    while ((int32_t)(ld_acquire_sys(my_pad + p) - e) < 0) {
      if (sm100::globaltimer() - t0 > kBarrierLimitNs) {
        atomicCAS(err, 0, code + p);
        return;
      }
    }
  }
}

struct DpArgs {
  float* const* grads;   // [world] flat fp32 gradient buffers (peer-mapped)
  bf16* const* shadows;  // [world] flat bf16 weight buffers (peer-mapped)
  float* master;         // local flat fp32 master weights (full size)
  float* m;              // shard-sized Adam state
  float* v;
  int64_t lo, n;         // shard [lo, lo + n), n a multiple of 4
  const float* lr;
  const int* step;
  AdamHyper h;
  int world;
  int clear;             // zero every rank's gradient shard after reading it (0: the next step's
                         // first micro-batch stores its gradients instead of adding)
};

template <int WORLD>
__global__ void __launch_bounds__(256) dp_fused_adamw_kernel(DpArgs a) {
  const float lr = *a.lr;
  const int t = *a.step;
  const float bc1 = 1.f - powf(a.h.b1, (float)t);
  const float bc2 = 1.f - powf(a.h.b2, (float)t);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * a.h.wd;
  const int world = WORLD > 0 ? WORLD : a.world;
  const int64_t n4 = a.n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gi = a.lo + 4 * i;
    float4 gs = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < world; ++p) {
      const float4 x = __ldcv(reinterpret_cast<const float4*>(a.grads[p] + gi));
      gs.x += x.x;
      gs.y += x.y;
      gs.z += x.z;
      gs.w += x.w;
    }
    if (a.clear) {
#pragma unroll 8
      for (int p = 0; p < world; ++p) __stcg(reinterpret_cast<float4*>(a.grads[p] + gi), make_float4(0.f, 0.f, 0.f, 0.f));
    }
    float4 pp = ld_f4(a.master + gi), mm = ld_f4(a.m + 4 * i), vv = ld_f4(a.v + 4 * i);
    float* pe = &pp.x;
    const float* ge = &gs.x;
    float* me = &mm.x;
    float* ve = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = ge[j] * a.h.grad_scale;
      me[j] = a.h.b1 * me[j] + (1.f - a.h.b1) * gj;
      ve[j] = a.h.b2 * ve[j] + (1.f - a.h.b2) * gj * gj;
      pe[j] = pe[j] * decay - step_size * me[j] / (sqrtf(ve[j]) * inv_sqrt_bc2 + a.h.eps);
    }
    st_f4(a.master + gi, pp);
    st_f4(a.m + 4 * i, mm);
    st_f4(a.v + 4 * i, vv);
    uint2 w;
    w.x = pack_bf16x2(pp.x, pp.y);
    w.y = pack_bf16x2(pp.z, pp.w);
#pragma unroll 8
    for (int p = 0; p < world; ++p) __stcg(reinterpret_cast<uint2*>(a.shadows[p] + gi), w);
  }
  __threadfence_system();
}

__device__ int g_dp_err = 0;

}  // namespace

// ---------------------------------------------------------------- IPC plumbing
cudaError_t ipc_alloc(size_t bytes, void** ptr, void* handle64) {
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return e;
  return cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle64), *ptr);
}
cudaError_t ipc_open(const void* handle64, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}
cudaError_t ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr); }
cudaError_t ipc_free(void* ptr) { return cudaFree(ptr); }

int* dp_err_word() {
  static std::atomic<int*> slots[64];
  return device_symbol_address(slots, g_dp_err);
}

int dp_error_code(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_dp_err, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_dp_err, &z, sizeof(int));
  }
  return v;
}

cudaError_t dp_barrier(uint32_t* const* pads_dev, uint32_t* my_pad, uint32_t* epoch, int rank, int world, int code,
                       cudaStream_t st) {
  dp_barrier_kernel<<<1, 32, 0, st>>>(pads_dev, my_pad, epoch, rank, world, dp_err_word(), code);
  return cudaGetLastError();
}

cudaError_t dp_fused_adamw(float* const* grads_dev, void* const* shadows_dev, float* master, float* m, float* v,
                           int64_t lo, int64_t n, const float* lr, const int* step, AdamHyper h, int world,
                           cudaStream_t st, int max_blocks, bool clear) {
  LLMT_REQUIRE(n % 4 == 0 && lo % 4 == 0, "dp_fused_adamw: shard bounds must be multiples of 4");
  if (n == 0) return cudaSuccess;
  DpArgs a{grads_dev, reinterpret_cast<bf16* const*>(shadows_dev), master, m, v, lo, n, lr, step, h, world, clear ? 1 : 0};
  // max_blocks > 0 keeps the kernel to a few SMs when it runs beside the backward
  const int64_t cap = max_blocks > 0 ? max_blocks : sm_count() * 4;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n / 4, 256), cap));
  switch (world) {
    case 2: dp_fused_adamw_kernel<2><<<grid, 256, 0, st>>>(a); break;
    case 4: dp_fused_adamw_kernel<4><<<grid, 256, 0, st>>>(a); break;
    case 8: dp_fused_adamw_kernel<8><<<grid, 256, 0, st>>>(a); break;
    default: dp_fused_adamw_kernel<0><<<grid, 256, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace llmt

// Shared device helpers for every llmt CUDA kernel (sm_100a only): vector load/store
// wrappers, bf16 conversion, warp reductions. No torch headers (see api.h).
#pragma once
#include <stdlib.h>

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

#include "../api.h"

// Argument check inside a launcher: records the message and returns cudaErrorInvalidValue.
#define LLMT_REQUIRE(cond, msg)          \
  do {                                   \
    if (!(cond)) {                       \
      ::llmt::set_last_error(msg);       \
      return cudaErrorInvalidValue;      \
    }                                    \
  } while (0)

namespace llmt {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

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

// Device address of a file-scope __device__ variable on the current device, looked up once per
// device and kept in `slots` (atomics: several host threads may make the first lookup at once;
// they store the same address).
template <typename T>
inline T* device_symbol_address(std::atomic<T*> (&slots)[64], const T& symbol) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  T* p = slots[dev].load(std::memory_order_relaxed);
  if (!p) {
    void* q = nullptr;
    if (cudaGetSymbolAddress(&q, symbol) != cudaSuccess) return nullptr;
    p = static_cast<T*>(q);
    slots[dev].store(p, std::memory_order_relaxed);
  }
  return p;
}

// ---------------------------------------------------------------- bounds-checked debug build
// Built with -DLLMT_DEBUG_BOUNDS=1 (the llmt._C_bounds module), every guarded global access
// first checks that the element range [lo, hi) it touches lies inside [0, n) of the buffer
// the launcher described. A range outside records the site and the first index in this
// translation unit's device word (first failure wins) and the access is skipped: nothing is
// read or written out of bounds, nothing traps, and the host reads the record with
// bounds_error(). In the release build LLMT_IN is `true` and compiles away.
#ifdef LLMT_DEBUG_BOUNDS
namespace bounds_detail {
static __device__ unsigned long long g_record = 0;  // one per translation unit
// bit 63 set | site << 40 | low 40 bits of the first index
static unsigned long long read_record(bool reset) {
  unsigned long long v = 0;
  cudaMemcpyFromSymbol(&v, g_record, sizeof(v));
  if (reset && v) {
    const unsigned long long z = 0;
    cudaMemcpyToSymbol(g_record, &z, sizeof(z));
  }
  return v;
}
static const int registered = ::llmt::register_bounds_reader(&read_record);
}  // namespace bounds_detail
__device__ __forceinline__ bool llmt_in_bounds(int64_t lo, int64_t hi, int64_t n, int site) {
  if (lo >= 0 && hi <= n && lo <= hi) return true;
  atomicCAS(&bounds_detail::g_record, 0ull,
            (1ull << 63) | ((unsigned long long)(site & 0x7fffff) << 40) | ((unsigned long long)lo & 0xffffffffffull));
  return false;
}
#define LLMT_IN(lo, hi, n, site) ::llmt::llmt_in_bounds((int64_t)(lo), (int64_t)(hi), (int64_t)(n), (site))
#else
#define LLMT_IN(lo, hi, n, site) true
#endif

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels on the training path are launched with programmatic stream serialisation: a kernel's
// CTAs may be scheduled while the previous kernel in the stream drains, and each kernel calls
// pdl_wait() before its first access to global memory, which blocks until the previous grid has
// completed and its writes are visible (so stream order is kept). pdl_trigger() lets the next
// kernel be scheduled once this CTA's main work is done. Inside a CUDA graph this removes most of
// the per-kernel launch gap.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Off unless LLMT_PDL=1: measured on the medium step (CUDA graph), programmatic launches made it
// 0.25 ms slower (16.63 vs 16.38 ms, 16.83 vs 16.56 ms in back-to-back pairs), the early-scheduled
// CTAs of the next kernel holding resources while they wait.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("LLMT_PDL");
    return e && e[0] == '1';
  }();
  return on;
}
// GEMM launches are programmatic by default (LLMT_PDL=0 turns them off, =1 makes every launch
// programmatic): the GEMM waits for its predecessor after its own set-up (barriers, TMEM,
// tensor-map prefetch), so that set-up overlaps the previous kernel's tail. Measured on the medium
// step in back-to-back pairs on one box: 14.39 / 14.31 / 14.40 ms against 14.51 / 14.48 / 14.49 ms.
inline bool pdl_gemm_enabled() {
  static const bool on = [] {
    const char* e = getenv("LLMT_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_if(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace llmt

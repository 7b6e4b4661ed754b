// Allocation-free RMSNorm backward: an entry point for callers that cannot allocate.
//
// This entry point has no counterpart in the reference project; it exists for callers that
// cannot call cudaMalloc (or any allocating routine) at the point where they run the
// backward: code inside a custom memory manager that owns every device byte, code running
// where allocation is forbidden by policy or would synchronise the device, and non-PyTorch
// hosts that link this library's C symbols without a caching allocator. Such callers still
// pass every input and output buffer; the kernel's only scratch (per-CTA partial sums of
// dw) lives in a fixed static device array compiled into the library.
//
//   int llmt_rmsnorm_bwd_noalloc(dy, s, w, rstd, ds_in, ds, ds16, dw, N, D, accumulate, stream)
//
// Same math and arguments as llmt::rmsnorm_bwd (norm.cu): dy bf16 (N, D), s fp32 (N, D),
// w fp32 (D), rstd fp32 (N), ds_in fp32 (N, D) or NULL, ds fp32 (N, D) out, ds16 bf16 (N, D)
// out or NULL, dw fp32 (D) written (accumulate = 0) or accumulated (accumulate = 1).
// Returns 0 (cudaSuccess) or a cudaError_t code; llmt_noalloc_last_error() explains argument
// errors. D must be a positive multiple of 8 and at most LLMT_NOALLOC_MAX_WIDTH (8192);
// larger widths are rejected with cudaErrorInvalidValue.
//
// Limits and sharing:
//  * The scratch array is LLMT_NOALLOC_SCRATCH_FLOATS floats (4 MiB) per GPU, held by every
//    GPU that loads the library until the process exits.
//  * Every call shares that one array and it keeps the last call's contents. The kernel
//    overwrites each partial row it reads before reading it, so nothing needs clearing, but
//    calls that overlap on the GPU (different streams, or different host threads without
//    ordering) race on it: serialise them, for example on one stream.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that first call
//    before any CUDA stream capture on that device. A first call made while its stream is
//    capturing is refused (cudaErrorStreamCaptureUnsupported, with a message). First calls
//    from several host threads at once are safe: the cache slots are atomics.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define LLMT_NOALLOC_SCRATCH_FLOATS (1 << 20)
#define LLMT_NOALLOC_MAX_WIDTH 8192

#ifdef __cplusplus
extern "C" {
#endif
int llmt_rmsnorm_bwd_noalloc(const void* dy_bf16, const float* s, const float* w, const float* rstd,
                             const float* ds_in, float* ds, void* ds16, float* dw, int64_t N, int D, int accumulate,
                             cudaStream_t stream);
const char* llmt_noalloc_last_error(void);
#ifdef __cplusplus
}
#endif

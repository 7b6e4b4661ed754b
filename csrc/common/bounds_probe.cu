// Self-test kernel of the bounds-checked build (compiled to nothing in the release build):
// one guarded store, so a test can show that an out-of-range index is recorded and skipped.
#include "common.cuh"

#ifdef LLMT_DEBUG_BOUNDS
namespace llmt {
namespace {
__global__ void bounds_probe_kernel(float* buf, int64_t n, int64_t i) {
  if (LLMT_IN(i, i + 1, n, 999)) buf[i] = 1.f;
}
}  // namespace

cudaError_t bounds_probe(float* buf, int64_t n, int64_t i, cudaStream_t st) {
  bounds_probe_kernel<<<1, 1, 0, st>>>(buf, n, i);
  return cudaGetLastError();
}
}  // namespace llmt
#endif

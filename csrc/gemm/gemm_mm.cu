// tcgen05 GEMM instantiations with MN-major A and B: wgrad (dW = dy^T x), contraction over
// tokens, fp32 output written or accumulated straight into the flat gradient buffer.
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static cudaError_t run_mm(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: return launch<BN, S, true, true, EPI_BF16>(mp, g, st);
    case EPI_F32: return launch<BN, S, true, true, EPI_F32>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for the dy^T x layout"); return cudaErrorInvalidValue;
  }
}

// CTA-pair (cta_group::2) 256 x 256 tiles
static cudaError_t run_mm_pair(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = kPairStages;
  switch (epi) {
    case EPI_BF16: return launch<256, S, true, true, EPI_BF16, 0, true>(mp, g, st);
    case EPI_F32: return launch<256, S, true, true, EPI_F32, 0, true>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for CTA pairs"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_mm(int bn, int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st, bool pair) {
  if (pair) return run_mm_pair(epi, mp, g, st);
  return bn == 256 ? run_mm<256>(epi, mp, g, st) : run_mm<128>(epi, mp, g, st);
}
}  // namespace llmt

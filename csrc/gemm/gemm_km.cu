// tcgen05 GEMM instantiations with K-major A and MN-major B: dgrad (dx = dy W), including
// the SwiGLU-backward epilogue of the w2 dgrad and the tensor-parallel dgrads whose rows go
// straight to their owner rank (PEER_RS).
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static cudaError_t run_km(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: return launch<BN, S, false, true, EPI_BF16>(mp, g, st);
    case EPI_F32: return launch<BN, S, false, true, EPI_F32>(mp, g, st);
    case EPI_SWIGLU_BWD: return launch<BN, S, false, true, EPI_SWIGLU_BWD>(mp, g, st);
    case EPI_PEER_RS: return launch<BN, S, false, true, EPI_PEER_RS>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for the dy W layout"); return cudaErrorInvalidValue;
  }
}

// CTA-pair (cta_group::2) 256 x 256 tiles
static cudaError_t run_km_pair(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = kPairStages;
  switch (epi) {
    case EPI_BF16: return launch<256, S, false, true, EPI_BF16, 0, true>(mp, g, st);
    case EPI_F32: return launch<256, S, false, true, EPI_F32, 0, true>(mp, g, st);
    case EPI_SWIGLU_BWD: return launch<256, S, false, true, EPI_SWIGLU_BWD, 0, true>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for CTA pairs"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_km(int bn, int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st, bool pair) {
  if (pair) return run_km_pair(epi, mp, g, st);
  return bn == 256 ? run_km<256>(epi, mp, g, st) : run_km<128>(epi, mp, g, st);
}
}  // namespace llmt

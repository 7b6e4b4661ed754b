// tcgen05 GEMM instantiations with K-major A and B: forward linears (y = x W^T) and the
// fused-epilogue GEMMs (SwiGLU, RoPE, cross-entropy).
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static cudaError_t run_kk(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: return launch<BN, S, false, false, EPI_BF16>(mp, g, st);
    case EPI_F32: return launch<BN, S, false, false, EPI_F32>(mp, g, st);
    case EPI_SWIGLU: return launch<BN, S, false, false, EPI_SWIGLU>(mp, g, st);
    case EPI_ROPE: return launch<BN, S, false, false, EPI_ROPE>(mp, g, st);
    case EPI_CE_FWD: return launch<BN, S, false, false, EPI_CE_FWD>(mp, g, st);
    case EPI_CE_BWD: return launch<BN, S, false, false, EPI_CE_BWD>(mp, g, st);
    case EPI_PEER_RS: return launch<BN, S, false, false, EPI_PEER_RS>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for the x W^T layout"); return cudaErrorInvalidValue;
  }
}

// CTA-pair (cta_group::2) 256 x 256 tiles
static cudaError_t run_kk_pair(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = kPairStages;
  switch (epi) {
    case EPI_BF16: return launch<256, S, false, false, EPI_BF16, 0, true>(mp, g, st);
    case EPI_F32: return launch<256, S, false, false, EPI_F32, 0, true>(mp, g, st);
    case EPI_SWIGLU: return launch<256, S, false, false, EPI_SWIGLU, 0, true>(mp, g, st);
    case EPI_ROPE: return launch<256, S, false, false, EPI_ROPE, 0, true>(mp, g, st);
    case EPI_CE_FWD: return launch<256, S, false, false, EPI_CE_FWD, 0, true>(mp, g, st);
    case EPI_CE_BWD: return launch<256, S, false, false, EPI_CE_BWD, 0, true>(mp, g, st);
    case EPI_PEER_RS: return launch<256, S, false, false, EPI_PEER_RS, 0, true>(mp, g, st);
    default: set_last_error("gemm: epilogue not built for CTA pairs"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_kk(int bn, int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st, bool pair) {
  if (pair) return run_kk_pair(epi, mp, g, st);
  return bn == 256 ? run_kk<256>(epi, mp, g, st) : run_kk<128>(epi, mp, g, st);
}
}  // namespace llmt

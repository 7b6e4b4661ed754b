// tcgen05 GEMM instantiations with K-major A and B: forward linears (y = x W^T) and the
// fused-epilogue GEMMs (SwiGLU, RoPE, cross-entropy).
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static cudaError_t run_kk(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: return launch<BN, S, false, false, EPI_BF16>(ta, tb, g, st);
    case EPI_F32: return launch<BN, S, false, false, EPI_F32>(ta, tb, g, st);
    case EPI_SWIGLU: return launch<BN, S, false, false, EPI_SWIGLU>(ta, tb, g, st);
    case EPI_ROPE: return launch<BN, S, false, false, EPI_ROPE>(ta, tb, g, st);
    case EPI_CE_FWD: return launch<BN, S, false, false, EPI_CE_FWD>(ta, tb, g, st);
    case EPI_CE_BWD: return launch<BN, S, false, false, EPI_CE_BWD>(ta, tb, g, st);
    default: set_last_error("gemm: epilogue not built for the x W^T layout"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_kk(int bn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g,
                           cudaStream_t st) {
  return bn == 256 ? run_kk<256>(epi, ta, tb, g, st) : run_kk<128>(epi, ta, tb, g, st);
}
}  // namespace llmt

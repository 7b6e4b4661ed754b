// tcgen05 GEMM instantiations with K-major A and B: forward linears (y = x W^T) and the
// fused-epilogue GEMMs (SwiGLU, RoPE, cross-entropy).
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static void run_kk(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: launch<BN, S, false, false, EPI_BF16>(ta, tb, g); break;
    case EPI_F32: launch<BN, S, false, false, EPI_F32>(ta, tb, g); break;
    case EPI_SWIGLU: launch<BN, S, false, false, EPI_SWIGLU>(ta, tb, g); break;
    case EPI_ROPE: launch<BN, S, false, false, EPI_ROPE>(ta, tb, g); break;
    case EPI_CE_FWD: launch<BN, S, false, false, EPI_CE_FWD>(ta, tb, g); break;
    case EPI_CE_BWD: launch<BN, S, false, false, EPI_CE_BWD>(ta, tb, g); break;
    default: TORCH_CHECK(false, "llmt: epilogue ", epi, " not built for the x W^T layout");
  }
}

void gemm_launch_kk(int bn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  if (bn == 256) run_kk<256>(epi, ta, tb, g);
  else run_kk<128>(epi, ta, tb, g);
}
}  // namespace llmt

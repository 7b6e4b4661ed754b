// tcgen05 GEMM instantiations with K-major A and MN-major B: dgrad (dx = dy W), including
// the SwiGLU-backward epilogue of the w2 dgrad.
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static void run_km(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: launch<BN, S, false, true, EPI_BF16>(ta, tb, g); break;
    case EPI_F32: launch<BN, S, false, true, EPI_F32>(ta, tb, g); break;
    case EPI_SWIGLU_BWD: launch<BN, S, false, true, EPI_SWIGLU_BWD>(ta, tb, g); break;
    default: TORCH_CHECK(false, "llmt: epilogue ", epi, " not built for the dy W layout");
  }
}

void gemm_launch_km(int bn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  if (bn == 256) run_km<256>(epi, ta, tb, g);
  else run_km<128>(epi, ta, tb, g);
}
}  // namespace llmt

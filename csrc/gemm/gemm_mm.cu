// tcgen05 GEMM instantiations with MN-major A and B: wgrad (dW = dy^T x), contraction over
// tokens, fp32 output written or accumulated straight into the flat gradient buffer.
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static void run_mm(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: launch<BN, S, true, true, EPI_BF16>(ta, tb, g); break;
    case EPI_F32: launch<BN, S, true, true, EPI_F32>(ta, tb, g); break;
    default: TORCH_CHECK(false, "llmt: epilogue ", epi, " not built for the dy^T x layout");
  }
}

void gemm_launch_mm(int bn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g) {
  if (bn == 256) run_mm<256>(epi, ta, tb, g);
  else run_mm<128>(epi, ta, tb, g);
}
}  // namespace llmt

// tcgen05 GEMM instantiations for e4m3 operands (kind::f8f6f4), both K-major: the forward,
// dgrad and wgrad GEMMs of the fp8 linears, which read transposed fp8 copies where the bf16
// path reads an operand MN-major.
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int BN>
static cudaError_t run_f8(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  switch (epi) {
    case EPI_BF16: return launch<BN, S, false, false, EPI_BF16, 1>(mp, g, st);
    case EPI_F32: return launch<BN, S, false, false, EPI_F32, 1>(mp, g, st);
    case EPI_SWIGLU: return launch<BN, S, false, false, EPI_SWIGLU, 1>(mp, g, st);
    case EPI_SWIGLU_BWD: return launch<BN, S, false, false, EPI_SWIGLU_BWD, 1>(mp, g, st);
    case EPI_ROPE: return launch<BN, S, false, false, EPI_ROPE, 1>(mp, g, st);
    default: set_last_error("gemm_fp8: epilogue not built for e4m3 operands"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_f8(int bn, int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  return bn == 256 ? run_f8<256>(epi, mp, g, st) : run_f8<128>(epi, mp, g, st);
}
}  // namespace llmt

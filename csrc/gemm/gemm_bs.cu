// tcgen05 GEMM instantiations for block-scaled operands: MXFP8 (kind::mxf8f6f4.block_scale,
// e4m3 data, ue8m0 scale per 32) and NVFP4 (kind::mxf4nvf4.block_scale.block16, e2m1 data,
// ue4m3 scale per 16). Tiles are 128 x 128 (the scale chunks cover 128 rows) with five stages.
#include "gemm_kernel.cuh"

namespace llmt {
using namespace gemm_detail;

template <int KIND>
static cudaError_t run_bs(int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  constexpr int S = 5;
  switch (epi) {
    case EPI_BF16: return launch<128, S, false, false, EPI_BF16, KIND>(mp, g, st);
    case EPI_F32: return launch<128, S, false, false, EPI_F32, KIND>(mp, g, st);
    case EPI_SWIGLU: return launch<128, S, false, false, EPI_SWIGLU, KIND>(mp, g, st);
    case EPI_SWIGLU_BWD: return launch<128, S, false, false, EPI_SWIGLU_BWD, KIND>(mp, g, st);
    case EPI_ROPE: return launch<128, S, false, false, EPI_ROPE, KIND>(mp, g, st);
    default: set_last_error("gemm_bs: epilogue not built for block-scaled operands"); return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_launch_bs(int kind, int epi, const GemmMaps& mp, const GemmArgs& g, cudaStream_t st) {
  return kind == 3 ? run_bs<3>(epi, mp, g, st) : run_bs<2>(epi, mp, g, st);
}
}  // namespace llmt

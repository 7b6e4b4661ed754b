// Host entry of the tcgen05 GEMM: operand validation, TMA tensor maps, tile-width choice,
// dispatch to the per-layout instantiations (gemm_kk.cu, gemm_km.cu, gemm_mm.cu), and the
// per-row combine of the cross-entropy epilogue's partials.
#include "gemm_kernel.cuh"

namespace llmt {

namespace {
__device__ int g_gemm_err = 0;  // sticky: first bounded-wait timeout code seen by any GEMM launch

// Estimated time ~ waves x tile width; ties go to the wider (more efficient) tile.
int pick_bn(int M, int N, int epi) {
  if (epi == EPI_SWIGLU) return N >= 512 ? 256 : 128;
  if (epi == EPI_ROPE) return 128;
  const int64_t mb = cdiv(M, kGemmBM);
  const int64_t t128 = cdiv(mb * cdiv(N, 128), sm_count()) * 1;
  const int64_t t256 = cdiv(mb * cdiv(N, 256), sm_count()) * 2;
  return t256 <= t128 ? 256 : 128;
}

void* opt_ptr(const c10::optional<at::Tensor>& t) { return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr; }
}  // namespace

int* gemm_err_word() {
  static int* p = nullptr;
  if (!p) C10_CUDA_CHECK(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_gemm_err));
  return p;
}

int gemm_error_code(bool reset) {
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(int)));
  if (reset) {
    int z = 0;
    C10_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(int)));
  }
  return v;
}

// out = op(a) @ op(b) with op = transpose when ta/tb. a, b bf16 row-major with unit inner
// stride; every row pitch a multiple of 16 bytes and every base 16-byte aligned (TMA rules,
// checked here before any tensor map is built). epi selects the fused epilogue.
void gemm(at::Tensor a, at::Tensor b, bool ta, bool tb, int64_t epi, at::Tensor out, bool accumulate,
          c10::optional<at::Tensor> aux, c10::optional<at::Tensor> out2, int64_t split,
          c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t, int64_t T, int64_t hd, int64_t rot_cols,
          c10::optional<at::Tensor> tgt, c10::optional<at::Tensor> lse, c10::optional<at::Tensor> grad_out,
          c10::optional<at::Tensor> part, c10::optional<at::Tensor> tlogit, double alpha, int64_t bn) {
  LLMT_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm operands must be CUDA tensors");
  LLMT_CHECK_DTYPE(a, at::kBFloat16);
  LLMT_CHECK_DTYPE(b, at::kBFloat16);
  LLMT_CHECK(a.dim() == 2 && b.dim() == 2, "gemm operands must be 2D");
  LLMT_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm operands need unit inner stride");
  LLMT_CHECK(tma_ok(a.data_ptr(), a.stride(0), 2), "gemm: a must be 16-byte aligned with a 16-byte-multiple row pitch");
  LLMT_CHECK(tma_ok(b.data_ptr(), b.stride(0), 2), "gemm: b must be 16-byte aligned with a 16-byte-multiple row pitch");
  LLMT_CHECK(!(ta && tb), "gemm: a^T b^T is not a supported layout");
  const int M = ta ? a.size(1) : a.size(0);
  const int K = ta ? a.size(0) : a.size(1);
  int N = tb ? b.size(0) : b.size(1);
  const int Kb = tb ? b.size(1) : b.size(0);
  LLMT_CHECK(K == Kb, "gemm inner dims differ: ", K, " vs ", Kb);
  if (epi == EPI_SWIGLU) {
    LLMT_CHECK(tb && b.size(0) == 2 * split, "SWIGLU gemm: b must be W13 (2*ffn, K)");
    N = (int)split;
  }
  LLMT_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  LLMT_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const int BN = bn ? (int)bn : pick_bn(M, N, (int)epi);
  LLMT_CHECK(BN == 128 || BN == 256, "gemm: BN must be 128 or 256");

  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.m_blocks = (int)cdiv(M, kGemmBM);
  g.n_blocks = (int)cdiv(N, epi == EPI_SWIGLU ? BN / 2 : BN);
  g.k_blocks = (int)cdiv(K, kGemmBK);
  g.out = out.data_ptr();
  g.ldo = out.dim() == 2 ? out.stride(0) : N;
  g.accumulate = accumulate ? 1 : 0;
  g.split = (int)split;
  g.alpha = (float)alpha;
  g.err = gemm_err_word();
  if (aux.has_value() && aux->defined()) {
    g.aux = aux->data_ptr();
    g.ld_aux = aux->stride(0);
  }
  if (out2.has_value() && out2->defined()) {
    g.out2 = out2->data_ptr();
    g.ldo2 = out2->stride(0);
  }
  g.cos_t = static_cast<const float*>(opt_ptr(cos_t));
  g.sin_t = static_cast<const float*>(opt_ptr(sin_t));
  g.T = (int)T;
  g.hd = (int)hd;
  g.rot_cols = (int)rot_cols;
  g.tgt = static_cast<const int64_t*>(opt_ptr(tgt));
  g.lse = static_cast<const float*>(opt_ptr(lse));
  g.grad_out = static_cast<const float*>(opt_ptr(grad_out));
  g.part = static_cast<float*>(opt_ptr(part));
  g.tlogit = static_cast<float*>(opt_ptr(tlogit));
  switch (epi) {
    case EPI_BF16: case EPI_ROPE: case EPI_CE_BWD: case EPI_SWIGLU:
      LLMT_CHECK_DTYPE(out, at::kBFloat16);
      LLMT_CHECK(out.dim() == 2 && out.size(0) >= M && out.size(1) >= N && out.stride(1) == 1 && out.stride(0) % 8 == 0,
                 "gemm: bf16 output must be (M, N) row-major with a 16-byte-multiple pitch");
      break;
    case EPI_F32:
      LLMT_CHECK_DTYPE(out, at::kFloat);
      LLMT_CHECK(out.dim() == 2 && out.size(0) >= M && out.size(1) >= N && out.stride(1) == 1 && out.stride(0) % 4 == 0,
                 "gemm: fp32 output must be (M, N) row-major with a 16-byte-multiple pitch");
      break;
    default: break;
  }
  if (epi == EPI_ROPE) LLMT_CHECK(g.cos_t && g.sin_t && hd % 64 == 0 && BN % hd == 0 && N % hd == 0 && T > 0, "ROPE gemm args");
  if (epi == EPI_SWIGLU) LLMT_CHECK(g.aux && aux->stride(0) % 8 == 0, "SWIGLU gemm needs the gu save buffer");
  if (epi == EPI_SWIGLU_BWD) LLMT_CHECK(g.aux && g.out2 && split == N, "SWIGLU_BWD gemm args");
  if (epi == EPI_CE_FWD) {
    LLMT_CHECK(g.tgt && g.part && g.tlogit, "CE_FWD gemm args");
    LLMT_CHECK(part->numel() >= (int64_t)M * g.n_blocks * 2, "CE_FWD partial buffer too small");
  }
  if (epi == EPI_CE_BWD) LLMT_CHECK(g.tgt && g.lse, "CE_BWD gemm args");

  const auto dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  alignas(64) CUtensorMap tmA;
  alignas(64) CUtensorMap tmB;
  if (!ta) make_tmap_2d(&tmA, a.data_ptr(), dt, 2, K, M, a.stride(0), kGemmBK, kGemmBM);
  else make_tmap_2d(&tmA, a.data_ptr(), dt, 2, M, K, a.stride(0), 64, kGemmBK);
  if (tb) {
    const int rows = epi == EPI_SWIGLU ? 2 * N : N;
    make_tmap_2d(&tmB, b.data_ptr(), dt, 2, K, rows, b.stride(0), kGemmBK, epi == EPI_SWIGLU ? BN / 2 : BN);
  } else {
    make_tmap_2d(&tmB, b.data_ptr(), dt, 2, N, K, b.stride(0), 64, kGemmBK);
  }
  if (!ta && tb) gemm_launch_kk(BN, (int)epi, tmA, tmB, g);
  else if (!ta && !tb) gemm_launch_km(BN, (int)epi, tmA, tmB, g);
  else gemm_launch_mm(BN, (int)epi, tmA, tmB, g);
}

namespace {
// Per-row combine of the CE_FWD partials into lse and loss = lse - target logit.
__global__ void ce_combine_kernel(const float* __restrict__ part, const float* __restrict__ tlogit,
                                  const int64_t* __restrict__ tgt, float* __restrict__ lse, float* __restrict__ loss,
                                  int M, int nblk, int V) {
  const int row = blockIdx.x * blockDim.y + threadIdx.y;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nblk; i += 32) {
    const float pm = part[((int64_t)row * nblk + i) * 2], ps = part[((int64_t)row * nblk + i) * 2 + 1];
    if (pm == -INFINITY) continue;
    const float nm = fmaxf(m, pm);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + ps * __expf(pm - nm);
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, m2);
    if (nm == -INFINITY) continue;
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - nm));
    m = nm;
  }
  if (threadIdx.x == 0) {
    const float l = m + logf(s);
    lse[row] = l;
    const int64_t t = tgt[row];
    loss[row] = (t >= 0 && t < V) ? l - tlogit[row] : 0.f;
  }
}
}  // namespace

void ce_combine(at::Tensor part, at::Tensor tlogit, at::Tensor tgt, at::Tensor lse, at::Tensor loss, int64_t nblk,
                int64_t V) {
  const int M = lse.numel();
  if (M == 0) return;
  dim3 block(32, 8);
  ce_combine_kernel<<<cdiv(M, 8), block, 0, cur_stream()>>>(part.data_ptr<float>(), tlogit.data_ptr<float>(),
                                                            tgt.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                                            loss.data_ptr<float>(), M, (int)nblk, (int)V);
  LLMT_LAUNCH_CHECK();
}

}  // namespace llmt

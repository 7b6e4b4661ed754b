// Host entry of the tcgen05 GEMM: operand validation, TMA tensor maps, tile-width choice,
// dispatch to the per-layout instantiations (gemm_kk.cu, gemm_km.cu, gemm_mm.cu), and the
// per-row combine of the cross-entropy epilogue's partials.
#include <string.h>

#include <stdio.h>

#include "gemm_kernel.cuh"

namespace llmt {

namespace {
__device__ int g_gemm_err = 0;  // sticky: first bounded-wait timeout code seen by any GEMM launch

int* gemm_err_word() {
  static std::atomic<int*> slots[64];
  return device_symbol_address(slots, g_gemm_err);
}
}  // namespace

// CTA-pair tiles are on unless LLMT_GEMM_PAIRS=0 (kept for measurements).
static bool gemm_pairs_enabled() {
  static const bool on = [] {
    const char* e = getenv("LLMT_GEMM_PAIRS");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Estimated time ~ waves x tile width; ties go to the wider (more efficient) tile.
int gemm_pick_bn(int M, int N, int epi) {
  if (epi == EPI_SWIGLU) return N >= 512 ? 256 : 128;
  const int64_t mb = cdiv(M, kGemmBM);
  const int64_t t128 = cdiv(mb * cdiv(N, 128), persistent_sms()) * 1;
  const int64_t t256 = cdiv(mb * cdiv(N, 256), persistent_sms()) * 2;
  return t256 <= t128 ? 256 : 128;
}

// Tile width and split-K from a wave model: cost = waves x (k-blocks per unit + fixed
// per-unit overhead) x tile width; splits only when the output is an fp32 reduce-add.
void gemm_plan(int M, int N, int K, int epi, bool can_split, int* bn, int* splits) {
  const int sms = persistent_sms();
  const int64_t mb = cdiv(M, kGemmBM), kb = cdiv(K, kGemmBK);
  double best = 1e30;
  *bn = gemm_pick_bn(M, N, epi);
  *splits = 1;
  for (int BN : {128, 256}) {
    if (epi == EPI_SWIGLU) BN = *bn;
    if (epi == EPI_ROPE && BN % 128) continue;
    const int64_t tiles = mb * cdiv(N, epi == EPI_SWIGLU ? BN / 2 : BN);
    const int smax = can_split ? (int)std::min<int64_t>(16, std::max<int64_t>(1, kb / 4)) : 1;
    for (int s = 1; s <= smax; ++s) {
      const int64_t kps = cdiv(kb, s);
      const int64_t units = tiles * cdiv(kb, kps);
      // BN=128 tiles reach ~70% of the BN=256 per-FLOP rate (operand smem bandwidth). A split
      // pays for its reduce-add traffic and for clearing the output first: measured on the
      // medium weight gradients (K 4096), 1.3x per unit plus a fixed 10 units (~2 us)
      const double cost = (double)cdiv(units, sms) * (double)(kps + 3) * (BN == 256 ? 2.0 : 1.45) * (s > 1 ? 1.3 : 1.0) +
                          (s > 1 ? 10.0 : 0.0);
      if (cost < best - 1e-9) {
        best = cost;
        *bn = BN;
        *splits = (int)cdiv(kb, kps);
      }
    }
    if (epi == EPI_SWIGLU) break;
  }
}

int gemm_error_code(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(int));
  }
  return v;
}

// Epilogue output maps: 32x32 boxes, one per epilogue warp and chunk (see Stager).
static bool make_out_maps(int epi, const GemmArgs& g, int M, int N, GemmMaps* mp) {
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  switch (epi) {
    case EPI_F32:
      return make_tmap_2d(&mp->c, g.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, g.ldo, 32, 32,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    case EPI_BF16: case EPI_CE_BWD:  // 32 rows x 64 columns (128-byte rows)
      return make_tmap_2d(&mp->c, g.out, dt, 2, N, M, g.ldo, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    case EPI_ROPE:
      return make_tmap_2d(&mp->c, g.out, dt, 2, N, M, g.ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    case EPI_SWIGLU:
      return make_tmap_2d(&mp->c, g.out, dt, 2, N, M, g.ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
             make_tmap_3d(&mp->c2, g.aux, dt, 2, N, 2, M, N, g.ld_aux, 32, 1, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    case EPI_SWIGLU_BWD:  // c: the saved [g | u] rows (loaded), c2: [dg | du] (stored)
      return make_tmap_3d(&mp->c, g.aux, dt, 2, N, 2, M, N, g.ld_aux, 32, 1, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
             make_tmap_3d(&mp->c2, g.out2, dt, 2, N, 2, M, N, g.ldo2, 32, 1, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    default: return true;
  }
}

cudaError_t gemm(const void* a, int64_t lda, const void* b, int64_t ldb, bool ta, bool tb, int M, int N, int K,
                 int epi, int bn, GemmArgs g, cudaStream_t st, int force_splits) {
  LLMT_REQUIRE(!(ta && tb), "gemm: a^T b^T is not a supported layout");
  LLMT_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  LLMT_REQUIRE(N % 8 == 0, "gemm: N must be a multiple of 8");
  LLMT_REQUIRE(tma_ok(a, lda, 2) && tma_ok(b, ldb, 2), "gemm: operands need 16-byte aligned bases and row pitches");
  int BN = bn, splits = 1;
  const bool can_split = epi == EPI_F32 && g.accumulate;
  if (!BN) gemm_plan(M, N, K, epi, can_split, &BN, &splits);
  if (force_splits > 0) {
    LLMT_REQUIRE(force_splits == 1 || can_split, "gemm: split-K needs an fp32 reduce-add output");
    splits = force_splits;
  }
  LLMT_REQUIRE(BN == 128 || BN == 256, "gemm: BN must be 128 or 256");
  if (epi == EPI_PEER_RS)
    LLMT_REQUIRE(g.peer && g.rows_per_rank > 0 && M % g.rows_per_rank == 0 && N % 32 == 0 && g.ldo % 8 == 0 &&
                     !ta,
                 "gemm: PEER_RS needs peer slots, M a multiple of the rows per rank, N a multiple of 32");
  if (epi == EPI_ROPE) LLMT_REQUIRE(g.hd % 64 == 0 && BN % g.hd == 0 && N % g.hd == 0, "gemm: bad RoPE epilogue shape");
  if (g.ag_src) {
    LLMT_REQUIRE(!ta && (epi == EPI_BF16 || epi == EPI_ROPE || epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD),
                 "gemm: a fused all-gather needs a K-major A and a bf16 epilogue");
    LLMT_REQUIRE(g.ag_dst && g.ag_flags && g.ag_tp >= 1 && g.ag_tp <= 8 && g.tp_rank >= 0 && g.tp_rank < g.ag_tp,
                 "gemm: fused all-gather needs gather buffers, flags and 0 <= rank < tp <= 8");
    LLMT_REQUIRE(g.rows_per_rank > 0 && g.rows_per_rank % 128 == 0 && (int64_t)g.ag_tp * g.rows_per_rank == M,
                 "gemm: fused all-gather needs M = tp x rows per rank, rows per rank a multiple of 128");
    LLMT_REQUIRE(K % 8 == 0 && g.ag_lds % 8 == 0 && lda % 8 == 0 && (reinterpret_cast<uintptr_t>(g.ag_src) & 15) == 0,
                 "gemm: fused all-gather rows must be 16-byte aligned");
    g.ag_ldd = lda;
  }
  // 256 x 256 tiles on CTA pairs wherever the planner picked 256-wide tiles and M fills them
  const bool pair = BN == 256 && M > kGemmBM && gemm_pairs_enabled();
  g.M = M;
  g.N = N;
  g.K = K;
  g.m_blocks = (int)cdiv(M, pair ? 2 * kGemmBM : kGemmBM);
  g.n_blocks = (int)cdiv(N, epi == EPI_SWIGLU ? BN / 2 : BN);
  g.k_blocks = (int)cdiv(K, kGemmBK);
  g.k_per_split = (int)cdiv(g.k_blocks, splits);
  g.splits = (int)cdiv(g.k_blocks, g.k_per_split);
  g.err = gemm_err_word();
  // consecutive tiles share the larger operand's block: A (M x K) larger -> walk N, else walk M,
  // so the larger operand streams from DRAM once while the smaller stays in L2
  g.n_fastest = M > N ? 1 : 0;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  alignas(64) GemmMaps mp;
  memset(&mp, 0, sizeof(mp));
  const bool ok_a = ta ? make_tmap_2d(&mp.a, a, dt, 2, M, K, lda, 64, kGemmBK)
                       : make_tmap_2d(&mp.a, a, dt, 2, K, M, lda, kGemmBK, kGemmBM);
  if (g.ag_src)
    LLMT_REQUIRE(make_tmap_2d(&mp.a2, g.ag_src, dt, 2, K, g.rows_per_rank, g.ag_lds, kGemmBK, kGemmBM),
                 "gemm: fused all-gather: tensor map of this rank's rows rejected");
  const int code_a = last_tmap_result();
  bool ok_b;
  if (tb) {
    const int rows = epi == EPI_SWIGLU ? 2 * N : N;
    ok_b = make_tmap_2d(&mp.b, b, dt, 2, K, rows, ldb, kGemmBK, (epi == EPI_SWIGLU || pair) ? BN / 2 : BN);
  } else {
    ok_b = make_tmap_2d(&mp.b, b, dt, 2, N, K, ldb, 64, kGemmBK);
  }
  if (!ok_a || !ok_b) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "gemm: cuTensorMapEncodeTiled rejected operand %s (result %d; M=%d N=%d K=%d ta=%d tb=%d lda=%lld "
             "ldb=%lld a%%16=%d b%%16=%d epi=%d)",
             ok_a ? "B" : "A", ok_a ? last_tmap_result() : code_a, M, N, K, (int)ta, (int)tb, (long long)lda, (long long)ldb,
             (int)(reinterpret_cast<uintptr_t>(a) & 15), (int)(reinterpret_cast<uintptr_t>(b) & 15), epi);
    set_last_error(msg);
    return cudaErrorInvalidValue;
  }
  LLMT_REQUIRE(make_out_maps(epi, g, M, N, &mp), "gemm: output tensor map rejected (pitch/alignment)");
  if (!ta && tb) return gemm_launch_kk(BN, epi, mp, g, st, pair);
  if (!ta && !tb) return gemm_launch_km(BN, epi, mp, g, st, pair);
  return gemm_launch_mm(BN, epi, mp, g, st, pair);
}


cudaError_t gemm_fp8(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int epi, int bn,
                     GemmArgs g, cudaStream_t st, int force_splits) {
  LLMT_REQUIRE(M > 0 && N > 0 && K > 0, "gemm_fp8: empty problem");
  LLMT_REQUIRE(N % 8 == 0 && K % 16 == 0, "gemm_fp8: N must be a multiple of 8 and K of 16");
  LLMT_REQUIRE(tma_ok(a, lda, 1) && tma_ok(b, ldb, 1), "gemm_fp8: operands need 16-byte aligned bases and row pitches");
  LLMT_REQUIRE(g.scale_a && g.scale_b, "gemm_fp8: needs both inverse scales");
  LLMT_REQUIRE(epi == EPI_BF16 || epi == EPI_F32 || epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD || epi == EPI_ROPE,
               "gemm_fp8: epilogue not built for e4m3 operands");
  int BN = bn, splits = 1;
  const bool can_split = epi == EPI_F32 && g.accumulate;
  // a k-block is 128 e4m3 elements, the bytes of 64 bf16 ones: plan as K / 2 of bf16
  if (!BN) gemm_plan(M, N, (K + 1) / 2, epi, can_split, &BN, &splits);
  if (force_splits > 0) {
    LLMT_REQUIRE(force_splits == 1 || can_split, "gemm_fp8: split-K needs an fp32 reduce-add output");
    splits = force_splits;
  }
  LLMT_REQUIRE(BN == 128 || BN == 256, "gemm_fp8: BN must be 128 or 256");
  if (epi == EPI_ROPE)
    LLMT_REQUIRE(g.hd % 64 == 0 && BN % g.hd == 0 && N % g.hd == 0, "gemm_fp8: bad RoPE epilogue shape");
  constexpr int KE = 2 * kGemmBK;
  g.M = M;
  g.N = N;
  g.K = K;
  g.m_blocks = (int)cdiv(M, kGemmBM);
  g.n_blocks = (int)cdiv(N, epi == EPI_SWIGLU ? BN / 2 : BN);
  g.k_blocks = (int)cdiv(K, KE);
  g.k_per_split = (int)cdiv(g.k_blocks, splits);
  g.splits = (int)cdiv(g.k_blocks, g.k_per_split);
  g.err = gemm_err_word();
  // consecutive tiles share the larger operand's block: A (M x K) larger -> walk N, else walk M,
  // so the larger operand streams from DRAM once while the smaller stays in L2
  g.n_fastest = M > N ? 1 : 0;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  alignas(64) GemmMaps mp;
  memset(&mp, 0, sizeof(mp));
  const int rows_b = epi == EPI_SWIGLU ? 2 * N : N;
  const bool ok_a = make_tmap_2d(&mp.a, a, dt, 1, K, M, lda, KE, kGemmBM);
  const bool ok_b = ok_a && make_tmap_2d(&mp.b, b, dt, 1, K, rows_b, ldb, KE, epi == EPI_SWIGLU ? BN / 2 : BN);
  if (!ok_a || !ok_b) {
    char msg[200];
    snprintf(msg, sizeof(msg), "gemm_fp8: cuTensorMapEncodeTiled rejected operand %s (result %d; M=%d N=%d K=%d)",
             ok_a ? "B" : "A", last_tmap_result(), M, N, K);
    set_last_error(msg);
    return cudaErrorInvalidValue;
  }
  LLMT_REQUIRE(make_out_maps(epi, g, M, N, &mp), "gemm_fp8: output tensor map rejected (pitch/alignment)");
  return gemm_launch_f8(BN, epi, mp, g, st);
}


cudaError_t gemm_bs(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int epi,
                    GemmArgs g, cudaStream_t st, int force_splits) {
  LLMT_REQUIRE(kind == 2 || kind == 3, "gemm_bs: kind must be 2 (MXFP8) or 3 (NVFP4)");
  LLMT_REQUIRE(M > 0 && N > 0 && K > 0, "gemm_bs: empty problem");
  LLMT_REQUIRE(N % 8 == 0 && K % 32 == 0, "gemm_bs: N must be a multiple of 8 and K of 32");
  LLMT_REQUIRE(tma_ok(a, lda, 1) && tma_ok(b, ldb, 1), "gemm_bs: operands need 16-byte aligned bases and row pitches");
  LLMT_REQUIRE(g.sfa && g.sfb && (reinterpret_cast<uintptr_t>(g.sfa) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(g.sfb) & 15) == 0,
               "gemm_bs: needs 16-byte aligned scale-factor buffers");
  LLMT_REQUIRE(kind == 2 || (g.scale_a && g.scale_b), "gemm_bs: NVFP4 needs both per-tensor decode scales");
  LLMT_REQUIRE(epi == EPI_BF16 || epi == EPI_F32 || epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD || epi == EPI_ROPE,
               "gemm_bs: epilogue not built for block-scaled operands");
  constexpr int BN = 128;
  const int kbytes = kind == 3 ? K / 2 : K;  // row length of a and b in bytes
  const int k_blocks = (int)cdiv(kbytes, 2 * kGemmBK);
  int splits = 1;
  const bool can_split = epi == EPI_F32 && g.accumulate;
  if (force_splits > 0) {
    LLMT_REQUIRE(force_splits == 1 || can_split, "gemm_bs: split-K needs an fp32 reduce-add output");
    splits = force_splits;
  } else if (can_split) {
    int bn = 0;
    gemm_plan(M, N, kbytes / 2, epi, true, &bn, &splits);
  }
  if (epi == EPI_ROPE) LLMT_REQUIRE(g.hd % 64 == 0 && BN % g.hd == 0 && N % g.hd == 0, "gemm_bs: bad RoPE epilogue shape");
  if (epi == EPI_SWIGLU) LLMT_REQUIRE(N % 64 == 0, "gemm_bs: SwiGLU needs ffn a multiple of 64");
  g.M = M;
  g.N = N;
  g.K = K;
  g.m_blocks = (int)cdiv(M, kGemmBM);
  g.n_blocks = (int)cdiv(N, epi == EPI_SWIGLU ? BN / 2 : BN);
  g.k_blocks = k_blocks;
  g.k_per_split = (int)cdiv(k_blocks, splits);
  g.splits = (int)cdiv(k_blocks, g.k_per_split);
  g.sf_chunks = k_blocks * (kind == 2 ? 1 : 4);
  g.err = gemm_err_word();
  // consecutive tiles share the larger operand's block: A (M x K) larger -> walk N, else walk M,
  // so the larger operand streams from DRAM once while the smaller stays in L2
  g.n_fastest = M > N ? 1 : 0;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  alignas(64) GemmMaps mp;
  memset(&mp, 0, sizeof(mp));
  const int rows_b = epi == EPI_SWIGLU ? 2 * N : N;
  const bool ok_a = make_tmap_2d(&mp.a, a, dt, 1, kbytes, M, lda, 2 * kGemmBK, kGemmBM);
  const bool ok_b = ok_a && make_tmap_2d(&mp.b, b, dt, 1, kbytes, rows_b, ldb, 2 * kGemmBK, BN);
  if (!ok_a || !ok_b) {
    char msg[200];
    snprintf(msg, sizeof(msg), "gemm_bs: cuTensorMapEncodeTiled rejected operand %s (result %d; M=%d N=%d K=%d)",
             ok_a ? "B" : "A", last_tmap_result(), M, N, K);
    set_last_error(msg);
    return cudaErrorInvalidValue;
  }
  LLMT_REQUIRE(make_out_maps(epi, g, M, N, &mp), "gemm_bs: output tensor map rejected (pitch/alignment)");
  return gemm_launch_bs(kind, epi, mp, g, st);
}

namespace {
// Per-row combine of the CE_FWD partials into lse and loss = lse - target logit.
__global__ void ce_combine_kernel(const float* __restrict__ part, const float* __restrict__ tlogit,
                                  const int64_t* __restrict__ tgt, float* __restrict__ lse, float* __restrict__ loss,
                                  int M, int nblk, int V) {
  pdl_wait();
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

cudaError_t ce_combine(const float* part, const float* tlogit, const int64_t* tgt, float* lse, float* loss, int M,
                       int nblk, int V, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  dim3 block(32, 8);
  launch_pdl(ce_combine_kernel, (unsigned)cdiv(M, 8), block, 0, st, part, tlogit, tgt, lse, loss, M, nblk, V);
  return cudaGetLastError();
}

}  // namespace llmt

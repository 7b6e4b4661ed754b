// Persistent warp-specialized tcgen05/TMEM GEMM for sm_100a with fused epilogues.
//
// Replaces every cuBLAS GEMM of the reference step (bench_train.py:121-162 nn.Linear under
// autocast, kernels/triton_ops.py:383-390 lm-head chunks): forward y = x W^T, dgrad
// dx = dy W, wgrad dW = dy^T x, with fp32 accumulation in tensor memory.
//
//   D[M, N] (+)= A'[M, K] * B'[K, N]
//   A' = a (K-major) or a^T (MN-major); B' = b^T (K-major) or b (MN-major), all row-major
//   PyTorch tensors, so fwd/dgrad/wgrad never need a transposed copy.
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles (BM = 128, BN = 128|256, BK = 64):
//   warp 0    TMA producer: STAGES-deep ring of A/B tiles in 128B-swizzled shared memory
//   warp 1    TMEM allocator + single-thread tcgen05.mma issuer (4 x K=16 per stage)
//   warps 2-5 epilogue: tcgen05.ld 32x32b of the accumulator, fused math, global stores
// Two accumulators live in TMEM (2 x BN fp32 columns) so the epilogue of tile i overlaps the
// MMAs of tile i+1. No TMA multicast is used (the kernel also runs in multi-GPU jobs).
//
// Epilogues:
//   BF16       out = bf16(acc)
//   F32        out = acc (+ out when accumulating: fp32 main-grad accumulation)
//   SWIGLU     merged w1||w3 GEMM: the B tile holds BN/2 rows of W1 and the same BN/2 rows
//              of W3 (two TMA boxes), so acc = [g | u] for the same h columns;
//              writes h = silu(g) * u plus g and u (needed by the backward)
//   SWIGLU_BWD w2 dgrad: acc = dh; reads g, u and writes dg, du (reference triton_ops.py:182-194)
//   ROPE       qkv GEMM: rotate-half RoPE on q/k columns while storing the packed qkv rows
//   CE_FWD     lm head: per-row partial max / sum-exp over the tile's vocab columns and the
//              target logit; logits are never written (reference triton_ops.py:338-364)
//   CE_BWD     lm head recompute: dlogits = (exp(acc - lse) - onehot) * grad_out * alpha
#pragma once
#include "../common/common.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.h"

namespace llmt {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kEpiStageBytes = 4 * 2 * 4096;

// Host launchers, one translation unit per operand layout (keeps the build parallel).
struct GemmMaps {
  CUtensorMap a, b, c, c2;  // operands, main output, auxiliary output
  CUtensorMap a2;           // fused all-gather: this rank's own rows of A (GemmArgs::ag_src)
};
// pair: 256 x 256 tiles on CTA pairs (cta_group::2), BN must be 256
cudaError_t gemm_launch_kk(int bn, int epi, const GemmMaps& m, const GemmArgs& g, cudaStream_t st, bool pair);  // fwd
cudaError_t gemm_launch_km(int bn, int epi, const GemmMaps& m, const GemmArgs& g, cudaStream_t st, bool pair);  // dgrad
cudaError_t gemm_launch_mm(int bn, int epi, const GemmMaps& m, const GemmArgs& g, cudaStream_t st, bool pair);  // wgrad
cudaError_t gemm_launch_f8(int bn, int epi, const GemmMaps& m, const GemmArgs& g, cudaStream_t st);  // e4m3, K-major
cudaError_t gemm_launch_bs(int kind, int epi, const GemmMaps& m, const GemmArgs& g, cudaStream_t st);  // MX / NV

namespace gemm_detail {

using namespace sm100;

// sigmoid on the SFU: 2^(-x log2 e) and a reciprocal, both approximate hardware ops
__device__ __forceinline__ float sigm(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return r;
}

__device__ __forceinline__ void load_bf16x32(const bf16* src, float* v, int col0, int N) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (col0 + q * 8 < N) {
      bf16x8_to_float(*reinterpret_cast<const BF16x8*>(src + q * 8), v + q * 8);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q * 8 + j] = 0.f;
    }
  }
}

// Per-warp output staging: each epilogue warp owns 32 accumulator rows and two 4 KB shared
// buffers. A 32x32 chunk is written into a buffer in the TMA swizzle layout (64B swizzle for
// bf16 rows of 64 B, 128B swizzle for fp32 rows of 128 B: conflict-free for the 32 row
// writers) and leaves with one bulk-tensor store issued by lane 0. Out-of-range rows and
// columns are clipped by the TMA unit, so the stores need no masks.
struct Stager {
  uint8_t* base;
  int buf;
  int lane;
  uint64_t* bar;      // per-warp mbarrier for epilogue-side TMA loads
  uint32_t bar_phase;
  // TMA-load two 32x32 bf16 boxes (halves 0 and 1 of a 3D map) into base[0:2K] and base[2K:4K];
  // the caller's previous stores from that buffer must have been read (acquire_all first).
  __device__ __forceinline__ bool load_pair3d(const CUtensorMap* tm, int x, int y, int* err) {
    if (lane == 0) {
      bar_arrive_expect_tx(bar, 4096);
      tma_load_3d(base, tm, bar, x, 0, y);
      tma_load_3d(base + 2048, tm, bar, x, 1, y);
    }
    const bool ok = wait_bar(bar, bar_phase, err, 5);
    bar_phase ^= 1;
    return ok;
  }
  __device__ __forceinline__ void wait_all_reads() {
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }
  __device__ __forceinline__ void get_bf16(const uint8_t* b, float* v) const {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      bf16x8_to_float(*reinterpret_cast<const BF16x8*>(b + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)), v + u * 8);
  }
  __device__ __forceinline__ uint8_t* acquire() {
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    uint8_t* b = base + buf * 4096;
    buf ^= 1;
    return b;
  }
  __device__ __forceinline__ void put_bf16(uint8_t* b, const float* v) const {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<BF16x8*>(b + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) = float_to_bf16x8(v + u * 8);
  }
  // 32 rows x 64 bf16 columns (128-byte rows, 128B swizzle): unit u (columns 8u .. 8u + 7) of row
  // `lane` at unit u ^ (lane & 7); v holds the row's 64 values
  __device__ __forceinline__ void put_bf16x64(uint8_t* b, const float* v) const {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      *reinterpret_cast<BF16x8*>(b + lane * 128 + ((u ^ (lane & 7)) << 4)) = float_to_bf16x8(v + u * 8);
  }
  __device__ __forceinline__ void put_f32(uint8_t* b, const float* v) const {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      *reinterpret_cast<float4*>(b + lane * 128 + ((u ^ (lane & 7)) << 4)) =
          make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  }
  __device__ __forceinline__ void store2d(const CUtensorMap* tm, uint8_t* b, int x, int y, bool reduce = false) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (reduce) tma_reduce_add_2d(tm, b, x, y);
      else tma_store_2d(tm, b, x, y);
      bulk_commit();
    }
  }
  __device__ __forceinline__ void store3d(const CUtensorMap* tm, uint8_t* b, int x, int y, int z) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tm, b, x, y, z);
      bulk_commit();
    }
  }
  __device__ __forceinline__ void drain() {
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
};

__device__ __forceinline__ bool lane_is_zero(const Stager& st) { return st.lane == 0; }

// row: this thread's accumulator row; wrow: the warp's first row (TMA box origin).
// SC: e4m3 operands with tensorwise scales (or NVFP4 with per-tensor decode scales); every
// accumulator value is multiplied by the two scales before the epilogue's math.
template <int EPI, int BN, bool F8 = false>
__device__ __forceinline__ void epilogue_tile(uint32_t taddr, int row, int wrow, int nb, const GemmArgs& a,
                                              const CUtensorMap* tmC, const CUtensorMap* tmC2, Stager& st) {
  const bool rv = row < a.M;
  float sc = 1.f;
  if constexpr (F8) sc = __ldg(a.scale_a) * __ldg(a.scale_b);
  auto cvt = [sc](uint32_t x) { return F8 ? __uint_as_float(x) * sc : __uint_as_float(x); };
  if constexpr (EPI == EPI_BF16 || EPI == EPI_CE_BWD) {
    // 64 columns per staged box and TMA store (half the stores, fences and buffer waits of 32)
    float l = 0.f, scale = 0.f;
    int64_t t = -1;
    if constexpr (EPI == EPI_CE_BWD) {
      if (rv) {
        l = a.lse[row];
        t = a.tgt[row];
      }
      scale = a.alpha * (a.grad_out ? *a.grad_out : 1.f);
    }
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int col0 = nb * BN + c * 64;
      if (col0 >= a.N) break;  // uniform across the warp
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c * 64, r0);
      tmem_ld32(taddr + c * 64 + 32, r1);
      tmem_wait_ld();
      float v[64];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = cvt(r0[j]);
        v[32 + j] = cvt(r1[j]);
      }
      if constexpr (EPI == EPI_CE_BWD) {
#pragma unroll
        for (int j = 0; j < 64; ++j) v[j] = (__expf(v[j] - l) - ((int64_t)(col0 + j) == t ? 1.f : 0.f)) * scale;
      }
      uint8_t* b = st.acquire();
      st.put_bf16x64(b, v);
      st.store2d(tmC, b, col0, wrow);
    }
  } else if constexpr (EPI == EPI_F32) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col0 = nb * BN + c * 32;
      if (col0 >= a.N) break;  // uniform across the warp
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = cvt(r[j]);
      uint8_t* b = st.acquire();
      st.put_f32(b, v);
      st.store2d(tmC, b, col0, wrow, a.accumulate != 0);
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    const int F = a.split;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int col0 = nb * (BN / 2) + c * 32;
      if (col0 >= F) break;
      uint32_t rg[32], ru[32];
      tmem_ld32(taddr + c * 32, rg);
      tmem_ld32(taddr + BN / 2 + c * 32, ru);
      tmem_wait_ld();
      float g[32], u[32], h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        g[j] = cvt(rg[j]);
        u[j] = cvt(ru[j]);
        h[j] = g[j] * sigm(g[j]) * u[j];
      }
      uint8_t* b = st.acquire();
      st.put_bf16(b, h);
      st.store2d(tmC, b, col0, wrow);
      b = st.acquire();
      st.put_bf16(b, g);
      st.store3d(tmC2, b, col0, 0, wrow);
      b = st.acquire();
      st.put_bf16(b, u);
      st.store3d(tmC2, b, col0, 1, wrow);
    }
  } else if constexpr (EPI == EPI_PEER_RS) {
    // bf16 rows straight into their owner rank's reduce-scatter slot through NVLink. A thread
    // holds one accumulator row, so a per-thread store would write 16-byte pieces of 32 rows;
    // instead each 32 x 64 chunk is staged in the warp's shared-memory buffer (128B swizzle) and
    // leaves row by row: lanes 8k .. 8k + 7 write one row's 128 contiguous bytes, four rows per
    // store instruction.
    const int rpr = a.rows_per_rank;
    const int sub = st.lane >> 3, u = st.lane & 7;
    uint8_t* b = st.base;  // the warp's first 4 KB buffer (this epilogue issues no TMA stores)
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int col0 = nb * BN + c * 64;
      if (col0 >= a.N) break;  // uniform across the warp
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c * 64, r0);
      tmem_ld32(taddr + c * 64 + 32, r1);
      tmem_wait_ld();
      float v[64];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = cvt(r0[j]);
        v[32 + j] = cvt(r1[j]);
      }
      __syncwarp();  // every lane has read the previous chunk out of the buffer
      st.put_bf16x64(b, v);
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rl = it * 4 + sub;  // row within the warp's 32
        const int grow = wrow + rl;
        if (grow < a.M && col0 + 8 * u < a.N) {
          const int q = grow / rpr;
          bf16* dst = static_cast<bf16*>(a.peer[q]) + ((int64_t)a.tp_rank * rpr + (grow - q * rpr)) * a.ldo + col0 +
                      8 * u;
          __stcg(reinterpret_cast<uint4*>(dst), *reinterpret_cast<const uint4*>(b + rl * 128 + ((u ^ (rl & 7)) << 4)));
        }
      }
    }
    (void)row;  // (the rows are made visible to their owners once, after the last tile)
  } else if constexpr (EPI == EPI_SWIGLU_BWD) {
    // g and u arrive by TMA (3D map over the saved [g | u] rows) one chunk ahead, into the
    // warp's two 4 KB buffers; dg and du are written back in place and leave by TMA.
    const int nchunks = min(BN / 32, (int)cdiv(a.N - nb * BN, 32));
    auto issue = [&](int c) {
      uint8_t* b = st.base + (c & 1) * 4096;
      if (st.lane == 0) {
        bulk_wait_read<0>();  // the store that last used this buffer has read it
        bar_arrive_expect_tx(&st.bar[c & 1], 4096);
        tma_load_3d(b, tmC, &st.bar[c & 1], nb * BN + c * 32, 0, wrow);
        tma_load_3d(b + 2048, tmC, &st.bar[c & 1], nb * BN + c * 32, 1, wrow);
      }
    };
    if (nchunks > 0) issue(0);
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      const int col0 = nb * BN + c * 32;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      if (c + 1 < nchunks) issue(c + 1);
      uint8_t* b = st.base + (c & 1) * 4096;
      const bool ok = wait_bar(&st.bar[c & 1], (st.bar_phase >> (c & 1)) & 1, a.err, 5);
      st.bar_phase ^= 1u << (c & 1);
      float g[32], u[32], dg[32], du[32];
      st.get_bf16(b, g);
      st.get_bf16(b + 2048, u);
      tmem_wait_ld();
      if (!ok) break;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float d = cvt(r[j]);
        const float sg = sigm(g[j]);
        dg[j] = d * u[j] * sg * (1.f + g[j] * (1.f - sg));
        du[j] = d * g[j] * sg;
      }
      __syncwarp();  // every lane has read g, u before the buffer is overwritten
      st.put_bf16(b, dg);
      st.put_bf16(b + 2048, du);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane_is_zero(st)) {
        tma_store_3d(tmC2, b, col0, 0, wrow);
        tma_store_3d(tmC2, b + 2048, col0, 1, wrow);
        bulk_commit();
      }
    }
  } else if constexpr (EPI == EPI_ROPE) {
    // The tables duplicate their halves (cos[f] == cos[f + hd/2]), and every head of the tile
    // uses the same row of them: each 32-wide slice of the first half is loaded once per tile
    // and applied to all heads.
    const int hd = a.hd, half = hd / 2;
    const int tpos = rv ? row % a.T : 0;
    const float* cr = a.cos_t + (int64_t)tpos * hd;
    const float* sr = a.sin_t + (int64_t)tpos * hd;
#pragma unroll 1
    for (int j = 0; j < half / 32; ++j) {
      float cv[32], sv[32];
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        const float4 c4 = ld_f4(cr + j * 32 + 4 * e4), s4 = ld_f4(sr + j * 32 + 4 * e4);
        cv[4 * e4] = c4.x; cv[4 * e4 + 1] = c4.y; cv[4 * e4 + 2] = c4.z; cv[4 * e4 + 3] = c4.w;
        sv[4 * e4] = s4.x; sv[4 * e4 + 1] = s4.y; sv[4 * e4 + 2] = s4.z; sv[4 * e4 + 3] = s4.w;
      }
#pragma unroll 1
      for (int hl = 0; hl < BN / hd; ++hl) {
        const int c1 = hl * hd + j * 32;
        const int col1 = nb * BN + c1;
        if (col1 >= a.N) break;
        uint32_t r1[32], r2[32];
        tmem_ld32(taddr + c1, r1);
        tmem_ld32(taddr + c1 + half, r2);
        tmem_wait_ld();
        float x1[32], x2[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          x1[e] = cvt(r1[e]);
          x2[e] = cvt(r2[e]);
        }
        if (col1 < a.rot_cols) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float y1 = x1[e] * cv[e] - x2[e] * sv[e];
            const float y2 = x2[e] * cv[e] + x1[e] * sv[e];
            x1[e] = y1;
            x2[e] = y2;
          }
        }
        uint8_t* b = st.acquire();
        st.put_bf16(b, x1);
        st.store2d(tmC, b, col1, wrow);
        b = st.acquire();
        st.put_bf16(b, x2);
        st.store2d(tmC, b, col1 + half, wrow);
      }
    }
  } else if constexpr (EPI == EPI_CE_FWD) {
    const int64_t t = rv ? a.tgt[row] : -1;
    float m = -INFINITY, s = 0.f, tl = 0.f;
    bool has_t = false;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col0 = nb * BN + c * 32;
      if (col0 >= a.N) break;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = cvt(r[j]);
        if (col0 + j < a.N) cm = fmaxf(cm, x);
        if ((int64_t)(col0 + j) == t) {
          tl = x;
          has_t = true;
        }
      }
      float cs = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) cs += __expf(cvt(r[j]) - cm);
      const float nm = fmaxf(m, cm);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + cs * __expf(cm - nm);
      m = nm;
    }
    if (rv) {
      float* p = a.part + ((int64_t)row * a.n_blocks + nb) * 2;
      p[0] = m;
      p[1] = s;
      if (has_t) a.tlogit[row] = tl;
    }
  }
}

// ---------------------------------------------------------------- fused tensor-parallel all-gather
// (GemmArgs::ag_*). The copy runs on the epilogue warps before their first tile, so it overlaps
// the first tiles' MMAs; the producer waits, per 128-row block of A, for the pieces of the
// owning rank (acquire at system scope, then a proxy fence: the rows were written by generic
// stores, local or through NVLink, and are read by TMA).
// 1 s: below the 2 s of the pipeline's own mbarrier waits, so a missing peer is what runs out first
// (the MMA warp waiting on the stalled producer would otherwise record its own timeout)
constexpr uint64_t kAgWaitLimitNs = 1000000000ull;
constexpr int kAgWaitCode = 8;

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Epilogue warps of every CTA (t = 0..127): this rank's rows into every rank's gather buffer, in
// 16-row pieces strided over the grid. A piece is loaded once and stored to every destination:
// first the rank that needs it soonest (rank p walks its row blocks from its own onwards, p, p+1,
// ..., so this rank's rows are wanted next by rank - 1, then rank - 2, ...), this rank's own
// buffer last (only later kernels read it; this GEMM loads its own blocks from ag_src). Thread t
// owns row t / 8 of the piece and its 16-byte columns t % 8, t % 8 + 8, ...: no index division in
// the copy loop, 16 loads in flight per thread.
__device__ __forceinline__ void ag_store_rows(const GemmArgs& a, int t) {
  constexpr int PR = 128 / kAgPieces;  // rows per piece (16: 8 threads per row)
  constexpr int U = 16;
  constexpr int kMaxTp = 8;
  const int k16 = a.K / 8;
  const int blocks = a.rows_per_rank / 128;
  const int pieces = blocks * kAgPieces;
  const int64_t ls = a.ag_lds / 8, ld = a.ag_ldd / 8;
  const int gblk0 = a.tp_rank * blocks;
  const int rr = t >> 3, c0 = t & 7;
  uint4* dst[kMaxTp];
#pragma unroll
  for (int j = 0; j < kMaxTp; ++j)
    dst[j] = j < a.ag_tp ? reinterpret_cast<uint4*>(a.ag_dst[(a.tp_rank + 2 * a.ag_tp - 1 - j) % a.ag_tp]) : nullptr;
  for (int u = blockIdx.x; u < pieces; u += gridDim.x) {
    const int64_t lrow = (int64_t)u * PR + rr;
    const uint4* src = reinterpret_cast<const uint4*>(a.ag_src) + lrow * ls;
    const int64_t doff = ((int64_t)a.tp_rank * a.rows_per_rank + lrow) * ld;
    for (int q0 = c0; q0 < k16; q0 += 8 * U) {
      uint4 v[U];
#pragma unroll
      for (int e = 0; e < U; ++e)
        if (q0 + 8 * e < k16) v[e] = __ldg(src + q0 + 8 * e);
#pragma unroll
      for (int j = 0; j < kMaxTp; ++j) {
        if (j < a.ag_tp) {
#pragma unroll
          for (int e = 0; e < U; ++e)
            if (q0 + 8 * e < k16) __stcg(dst[j] + doff + q0 + 8 * e, v[e]);
        }
      }
    }
    __threadfence_system();  // this thread's stores are visible system-wide before the counts
    named_bar_sync(1, 128);  // every epilogue thread has stored and fenced its part of the piece
    if (t < a.ag_tp) red_release_sys_add(a.ag_flags[t] + gblk0 + u / kAgPieces, 1u);
  }
}

// Producer: wait until 128-row block `blk` of A holds its owner's rows for this call. A wait that
// runs out records kAgWaitCode and stops waiting for the rest of the launch (no hang).
__device__ __forceinline__ void ag_wait_block(const GemmArgs& a, const uint32_t* flags, int blk, bool& give_up) {
  if (!give_up) {
    const uint64_t t0 = globaltimer();
    uint32_t spin = 0;
    while ((int32_t)(ld_acquire_sys_u32(flags + blk) - a.ag_expect) < 0) {
      if ((++spin & 63u) == 0 && globaltimer() - t0 > kAgWaitLimitNs) {
        atomicCAS(a.err, 0, kAgWaitCode);
        give_up = true;
        break;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Output tile of a linear tile index; a fused all-gather starts at this rank's own row blocks
// (available first) by rotating the row-block index.
__device__ __forceinline__ void tile_mn(const GemmArgs& g, int rest, int rot, int& mb, int& nb) {
  mb = g.n_fastest ? rest / g.n_blocks : rest % g.m_blocks;
  nb = g.n_fastest ? rest % g.n_blocks : rest / g.m_blocks;
  if (rot) mb = (mb + rot) % g.m_blocks;
}

// KIND: 0 bf16, 1 e4m3 with tensorwise scales, 2 MXFP8, 3 NVFP4 (2 and 3: block-scaled MMA with
// the scale-factor chunks of each k-block loaded next to its A / B tiles and copied into TMEM).
// PAIR: a cluster of two CTAs computes each 256 x BN tile with cta_group::2 MMAs (bf16, BN =
// 256): each CTA loads its 128 rows of A and its BN/2 columns of B and holds its 128 rows of the
// accumulator; the leader issues the MMAs. Per SM that halves the B operand traffic from L2,
// which bounds the one-CTA kernel at BN = 256.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int KIND = 0, bool PAIR = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
            const __grid_constant__ CUtensorMap tmA2, const GemmArgs args) {
  constexpr int BM = kGemmBM, BK = kGemmBK;
  constexpr bool F8 = KIND != 0, BS = KIND >= 2;
  static_assert(!F8 || (!A_MN && !B_MN), "8-bit operands are K-major only");
  static_assert(!BS || BN == 128, "block-scaled tiles are 128 x 128");
  constexpr int KX = F8 ? 2 * BK : BK;  // tensor-map units per k-block: one 128-byte swizzled row
  static_assert(!PAIR || (KIND == 0 && BN == 256), "CTA pairs: bf16 operands, 256-wide tiles");
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // PAIR: this CTA's half of B
  constexpr int NCH = KIND == 2 ? 1 : 4;                // scale chunks per k-block and operand
  constexpr uint32_t SF_BYTES = BS ? 2 * NCH * 512 : 0;  // A and B chunks of one stage
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int TMEM_COLS = BS ? 512 : 2 * BN;           // block-scaled: scales at column 256 on
  constexpr uint32_t SF_COLS = 2 * NCH * 4;              // TMEM columns of one stage's scales
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sf_smem = smem + STAGES * STAGE_BYTES;  // per stage: A chunks then B chunks
  uint8_t* stage_out = sf_smem + STAGES * SF_BYTES;  // 4 warps x 2 x 4 KB epilogue staging
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + kEpiStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;  // [4 warps x 2] epilogue-warp TMA load barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 8);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int* err = args.err;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0: the leader (issues the MMAs)
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&tfull[b], 1);
      bar_init(&tempty[b], PAIR ? 8 : 128);  // PAIR: one arrival per epilogue warp of both CTAs
    }
    for (int b = 0; b < 8; ++b) bar_init(&ebar[b], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (KIND == 0 && args.ag_src) prefetch_tmap(&tmA2);
  }
  if (warp == 1) {
    if constexpr (PAIR) tmem_alloc_pair<TMEM_COLS>(tmem_slot);
    else tmem_alloc<TMEM_COLS>(tmem_slot);
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote arrival
  else __syncthreads();
  tc_fence_after();
  // with a programmatic launch the set-up above overlaps the previous kernel's tail; nothing of
  // global memory is touched before that kernel has completed
  pdl_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int mn_tiles = args.m_blocks * args.n_blocks;
  const int num_tiles = mn_tiles * args.splits;
  const int kpb = args.k_per_split;  // k-blocks per split (splits > 1 only with reduce-add output)
  // persistent unit: one CTA, or one CTA pair (tiles of 2 x BM rows)
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int TM = PAIR ? 2 * BM : BM;  // rows of one tile

  // fused all-gather (bf16 only): this rank's row blocks first
  const bool ag = KIND == 0 && args.ag_src != nullptr;
  const int ag_rot = ag ? (args.tp_rank * args.rows_per_rank) / TM : 0;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ag_ready = -1;
      bool ag_give_up = false;
      const uint32_t* ag_my_flags = ag ? args.ag_flags[args.tp_rank] : nullptr;
      for (int tile = unit0; tile < num_tiles && ok; tile += units) {
        const int rest = tile % mn_tiles, ks = tile / mn_tiles;
        int mb, nb;
        tile_mn(args, rest, ag_rot, mb, nb);
        const int k_lo = ks * kpb, k_hi = min(args.k_blocks, k_lo + kpb);
        // fused all-gather: this rank's own row blocks come straight from its rows (tmA2, no
        // wait); another rank's block is loaded from the gather buffer once its pieces arrived
        const CUtensorMap* tma = &tmA;
        int arow0 = 0;  // row of tma where this tile's A rows start, minus the tile's own offset
        if constexpr (KIND == 0) {
          const int arow = mb * TM + (int)rank * BM;  // first row of this CTA's A tile
          const int own0 = args.tp_rank * args.rows_per_rank;
          if (ag && arow >= own0 && arow < own0 + args.rows_per_rank) {
            tma = &tmA2;
            arow0 = own0;
          } else if (ag && arow < args.M && arow / BM != ag_ready) {
            ag_wait_block(args, ag_my_flags, arow / BM, ag_give_up);
            ag_ready = arow / BM;
          }
        }
        for (int kb = k_lo; kb < k_hi; ++kb) {
          if (!wait_bar(&empty[stage], phase ^ 1, err, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if constexpr (PAIR) {
            // both CTAs' halves land on the leader's barrier; the leader expects them all
            if (rank == 0) bar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
            const uint32_t fb = cluster_map(&full[stage], 0);
            const int k0 = kb * KX;
            const int row = mb * TM + (int)rank * BM;
            if constexpr (!A_MN) {
              tma_load_2d_pair(sa, tma, fb, k0, row - arow0);
            } else {
              tma_load_2d_pair(sa, &tmA, fb, row, k0);
              tma_load_2d_pair(sa + 8192, &tmA, fb, row + 64, k0);
            }
            if constexpr (!B_MN) {
              if constexpr (EPI == EPI_SWIGLU) {  // leader: W1 rows, peer: the same W3 rows
                tma_load_2d_pair(sb, &tmB, fb, k0, (rank ? args.split : 0) + nb * (BN / 2));
              } else {
                tma_load_2d_pair(sb, &tmB, fb, k0, nb * BN + (int)rank * (BN / 2));
              }
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_2d_pair(sb + j * 8192, &tmB, fb, nb * BN + (int)rank * (BN / 2) + j * 64, k0);
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          bar_arrive_expect_tx(&full[stage], STAGE_BYTES + SF_BYTES);
          const int k0 = kb * KX;
          if constexpr (BS) {
            uint8_t* sfs = sf_smem + stage * SF_BYTES;
            const int64_t ck = (int64_t)kb * NCH;
            bulk_load(sfs, args.sfa + ((int64_t)mb * args.sf_chunks + ck) * 512, NCH * 512, &full[stage]);
            bulk_load(sfs + NCH * 512, args.sfb + ((int64_t)nb * args.sf_chunks + ck) * 512, NCH * 512, &full[stage]);
          }
          if constexpr (!A_MN) {
            tma_load_2d(sa, tma, &full[stage], k0, mb * BM - arow0);
          } else {
            tma_load_2d(sa, &tmA, &full[stage], mb * BM, k0);
            tma_load_2d(sa + 8192, &tmA, &full[stage], mb * BM + 64, k0);
          }
          if constexpr (!B_MN) {
            if constexpr (EPI == EPI_SWIGLU && !BS) {
              tma_load_2d(sb, &tmB, &full[stage], k0, nb * (BN / 2));
              tma_load_2d(sb + (BN / 2) * 128, &tmB, &full[stage], k0, args.split + nb * (BN / 2));
            } else {
              tma_load_2d(sb, &tmB, &full[stage], k0, nb * BN);
            }
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full[stage], nb * BN + j * 64, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = KIND == 3 ? make_idesc_bs(BM, BN, 1, 0)
                                 : KIND == 2 ? make_idesc_bs(BM, BN, 0, 1)
                                 : F8        ? make_idesc_e4m3(BM, BN)
                                             : make_idesc_bf16(TM, BN, A_MN, B_MN);
      int stage = 0, buf = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      for (int tile = unit0; tile < num_tiles && ok; tile += units) {
        const int ks = tile / mn_tiles;
        const int k_lo = ks * kpb, k_hi = min(args.k_blocks, k_lo + kpb);
        if (!wait_bar(&tempty[buf], aphase ^ 1, err, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (int kb = k_lo; kb < k_hi; ++kb) {
          if (!wait_bar(&full[stage], phase, err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
          uint32_t t_sfa = 0, t_sfb = 0;
          if constexpr (BS) {
            // this stage's scale chunks into its own TMEM columns (the MMAs that read the
            // previous contents of these columns completed before the stage was refilled)
            const uint32_t s_sf = smem_u32(sf_smem + stage * SF_BYTES);
            t_sfa = tmem_base + 256 + stage * SF_COLS;
            t_sfb = t_sfa + NCH * 4;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
              tmem_cp_sf(t_sfa + 4 * c, make_plain_desc(s_sf + c * 512, 128));
              tmem_cp_sf(t_sfb + 4 * c, make_plain_desc(s_sf + (NCH + c) * 512, 128));
            }
          }
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad =
                A_MN ? make_sw128_desc(sa + k * 2048, 8192, 1024) : make_sw128_desc(sa + k * 32, 16, 1024);
            const uint64_t bd =
                B_MN ? make_sw128_desc(sb + k * 2048, 8192, 1024) : make_sw128_desc(sb + k * 32, 16, 1024);
            const uint32_t acc = (kb > k_lo || k > 0) ? 1u : 0u;
            if constexpr (KIND == 2) {
              // one ue8m0 scale per row per K = 32 instruction: byte k of the chunk's columns
              mma_mxf8(d, ad, bd, idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4), t_sfa | ((uint32_t)k << 30),
                       t_sfb | ((uint32_t)k << 30), acc);
            } else if constexpr (KIND == 3) {
              // four ue4m3 scales per row per K = 64 instruction: chunk k
              mma_nvf4(d, ad, bd, idesc, t_sfa + 4 * k, t_sfb + 4 * k, acc);
            } else if constexpr (F8) {
              mma_f8(d, ad, bd, idesc, acc);
            } else if constexpr (PAIR) {
              mma_f16_pair(d, ad, bd, idesc, acc);
            } else {
              mma_f16(d, ad, bd, idesc, acc);
            }
          }
          if constexpr (PAIR) mma_commit_pair(&empty[stage]);
          else mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) mma_commit_pair(&tfull[buf]);
        else mma_commit(&tfull[buf]);
        buf ^= 1;
        if (buf == 0) aphase ^= 1;
      }
    }
  } else {
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    Stager st{stage_out + (warp - 2) * 8192, 0, lane, &ebar[(warp - 2) * 2], 0u};
    int buf = 0;
    uint32_t aphase = 0;
    if constexpr (KIND == 0) {
      if (ag) ag_store_rows(args, (int)threadIdx.x - 64);
    }
    for (int tile = unit0; tile < num_tiles; tile += units) {
      const int rest = tile % mn_tiles;
      int mb, nb;
      tile_mn(args, rest, ag_rot, mb, nb);
      if (!wait_bar(&tfull[buf], aphase, err, 4)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + buf * BN + ((uint32_t)(q * 32) << 16);
      const int row0 = mb * TM + (int)rank * BM;  // first row of this CTA's accumulator
      epilogue_tile<EPI, BN, KIND == 1 || KIND == 3>(taddr, row0 + row_in_tile, row0 + q * 32, nb, args, &tmC, &tmC2, st);
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) bar_arrive_cluster(cluster_map(&tempty[buf], 0));
      } else {
        bar_arrive(&tempty[buf]);
      }
      buf ^= 1;
      if (buf == 0) aphase ^= 1;
    }
    // PEER_RS: every row this thread stored to a peer is visible system-wide before the flag
    // barrier that follows the GEMM releases the owners
    if constexpr (EPI == EPI_PEER_RS) __threadfence_system();
    st.drain();
  }
  pdl_trigger();  // this CTA is done: the next kernel in the stream may be scheduled
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the pair's MMAs have read both CTAs' shared memory
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair<TMEM_COLS>(tmem_base);
    else tmem_dealloc<TMEM_COLS>(tmem_base);
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int KIND = 0, bool PAIR = false>
cudaError_t launch(const GemmMaps& mp, const GemmArgs& args, cudaStream_t st) {
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, KIND, PAIR>;
  constexpr size_t sf = KIND >= 2 ? 2 * (KIND == 2 ? 1 : 4) * 512 : 0;
  constexpr size_t smem =
      STAGES * (kGemmBM * kGemmBK * 2 + (PAIR ? BN / 2 : BN) * kGemmBK * 2 + sf) + kEpiStageBytes + 1024 + 256;
  static_assert(smem <= 232448, "GEMM shared memory exceeds the per-CTA limit");
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = args.m_blocks * args.n_blocks * args.splits;
  if constexpr (PAIR) {
    int pairs = std::min(tiles, persistent_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_gemm_enabled() ? 2 : 1;
    if (args.ag_src) {
      // a fused all-gather needs every pair resident at once (the producers wait for rows that
      // other CTAs' epilogue warps store): no more pairs than the clusters that fit together
      // (one value per instantiation: every GPU of a job is a B200; atomic, since host threads
      // may launch concurrently)
      static std::atomic<int> fit_cache{0};
      int fit = fit_cache.load(std::memory_order_relaxed);
      if (!fit) {
        cfg.gridDim = dim3(2 * pairs);
        cudaError_t e = cudaOccupancyMaxActiveClusters(&fit, kern, &cfg);
        if (e != cudaSuccess || fit < 1) return e != cudaSuccess ? e : cudaErrorLaunchOutOfResources;
        fit_cache.store(fit, std::memory_order_relaxed);
      }
      pairs = std::min(pairs, fit);
      cfg.gridDim = dim3(2 * pairs);
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mp.a, mp.b, mp.c, mp.c2, mp.a2, args);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  const int grid = std::min(tiles, persistent_sms());
  launch_pdl_if(pdl_gemm_enabled(), kern, grid, kGemmThreads, smem, st, mp.a, mp.b, mp.c, mp.c2, mp.a2, args);
  return cudaGetLastError();
}

template <int BN>
constexpr int stages_for() {
  return BN == 256 ? 4 : 6;
}
// CTA pairs hold half of B per stage (32 KB stages): six fit beside the epilogue staging.
constexpr int kPairStages = 6;

}  // namespace gemm_detail
}  // namespace llmt

// Causal flash attention backward on tcgen05 tensor cores (sm_100a), with the RoPE backward
// and the packed-dqkv write fused into its epilogues.
//
// Replaces the backward of the reference's SDPA (autograd of bench_train.py:141-142, three
// launches, perf_model/roofline.py:234-236) and its RoPE backward kernel
// (kernels/triton_ops.py:256-287): the result is written straight into the packed
// dqkv rows (B*T, (H + 2*KV) * hd) that the qkv dgrad/wgrad GEMMs read.
//
// FlashAttention-2 style split (Dao 2023): one CTA per (batch, kv head, 128-key block) owns
// dK/dV in TMEM and walks every query block at or after its keys (causal) of every query
// head in its GQA group. Per step, with S^T, dP^T and the accumulators in TMEM:
//   S^T  = K Q^T,  dP^T = V dO^T                 (M = 128 keys)
//   P^T  = exp(scale S^T - lse),  dS^T = P^T (dP^T - D)   (one thread per key row)
//   dV  += P^T dO,  dK += dS^T Q                  (P^T, dS^T staged in swizzled smem)
//   dQ   = dS K  (dS^T read as an MN-major A operand) -> TMA reduce-add into fp32 dq_acc
// Eight compute warps: two per TMEM lane quadrant, each taking half of the columns.
// D = rowsum(dO * O) comes from a small pre-pass; a post-pass turns dq_acc into bf16 with
// the RoPE backward applied. dK gets its RoPE backward in this kernel's epilogue.
#include "../common/common.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.h"

namespace llmt {
int* attn_err_word();

namespace {

using namespace sm100;

constexpr int kBM = 128;  // keys per CTA
constexpr int kBN = 128;  // queries per step
constexpr int kBwdThreads = 320;  // TMA warp, MMA warp, 8 compute warps (2 per TMEM lane quadrant)
constexpr int kComputeThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;
// One exponential pair in kBwdPolyEvery runs as the FMA-pipe polynomial (ex2_poly), 0 = none: the
// SFU issues 16 exponentials per clock per SM, the four schedulers 128 FMA-pipe lanes.
constexpr int kBwdPolyEvery = 4;

struct AttnBwdArgs {
  const float* lse;   // (B, H, T) natural log
  const float* dsum;  // (B, H, T) rowsum(dO * O)
  float* dq_acc;      // (B*T, H*hd) fp32, pre-zeroed
  bf16* dqkv;         // (B*T, (H + 2*KV) * hd)
  const float* cos_t;
  const float* sin_t;
  int B, T, H, KV, ld_qkv, ld_dq;
  float scale, scale_log2;
  int causal;
  int* err;
};

__device__ __forceinline__ uint32_t sw_unit(int r, int u) {
  return (uint32_t)((u >> 3) * 16384 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

template <int HD>
struct BwdSmem {
  static constexpr int STAGES = HD == 64 ? 2 : 1;
  static constexpr uint32_t T_BYTES = 128 * HD * 2;  // one 128-row tile
  static constexpr uint32_t K_OFF = 0;
  static constexpr uint32_t V_OFF = K_OFF + T_BYTES;
  static constexpr uint32_t Q_OFF = V_OFF + T_BYTES;
  static constexpr uint32_t DO_OFF = Q_OFF + STAGES * T_BYTES;
  static constexpr uint32_t P_OFF = DO_OFF + STAGES * T_BYTES;
  static constexpr uint32_t DS_OFF = P_OFF + 128 * 128 * 2;
  static constexpr uint32_t VEC_OFF = DS_OFF + 128 * 128 * 2;  // per stage: lse (128) + D (128) floats
  static constexpr int EPI_BUFS = 1;                             // dQ staging buffers per compute warp
  static constexpr uint32_t STG_OFF = VEC_OFF + STAGES * 1024;   // 8 warps x EPI_BUFS x 4 KB (32x32 fp32)
  static constexpr uint32_t BAR_OFF = STG_OFF + 8 * EPI_BUFS * 4096;
  static constexpr uint32_t TOTAL = BAR_OFF + 256 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(kBwdThreads, 1)
flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                 const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dkv,
                 const AttnBwdArgs a) {
  pdl_wait();
  using L = BwdSmem<HD>;
  constexpr int ST = L::STAGES;
  constexpr int TMEM_COLS = 512;
  constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 256 + HD;
  constexpr uint32_t C_DQ = HD == 64 ? 384 : 0;  // HD=128: dQ reuses S^T's columns
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;     // [ST]
  uint64_t* q_empty = bars + 3;    // [ST]
  uint64_t* s_full = bars + 5;
  uint64_t* pds_full = bars + 6;   // 128 arrivals
  uint64_t* pds_empty = bars + 7;
  uint64_t* dq_full = bars + 8;
  uint64_t* tm_free = bars + 9;    // 128 arrivals: S/dP/dQ columns free again
  uint64_t* dkv_full = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // blocks launch x-fastest: every (batch, kv head) of key block 0 first, so the longest causal
  // CTAs (low key blocks walk the most query blocks) start in the first wave and the short ones
  // fill in behind them
  const int bk = blockIdx.x;             // b * KV + kv head
  const int kb = blockIdx.y;             // key block
  const int b = bk / a.KV, kvh = bk % a.KV;
  const int group = a.H / a.KV;
  const int nqb = (int)cdiv(a.T, kBN);
  const int i_start = a.causal ? kb : 0;
  const int n_i = nqb - i_start;
  const int n_items = group * n_i;
  const int row0 = b * a.T;
  const int k0 = kb * kBM;
  int* err = a.err;

  if (threadIdx.x == 0) {
    bar_init(kv_full, 1);
    for (int s = 0; s < ST; ++s) {
      bar_init(&q_full[s], 1);
      bar_init(&q_empty[s], 1);
    }
    bar_init(s_full, 1);
    bar_init(pds_full, kComputeThreads);
    bar_init(pds_empty, 1);
    bar_init(dq_full, 1);
    bar_init(tm_free, kComputeThreads);
    bar_init(dkv_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv);
      prefetch_tmap(&tm_do);
      const int kcol = (a.H + kvh) * HD, vcol = (a.H + a.KV + kvh) * HD;
      bar_arrive_expect_tx(kv_full, 2 * L::T_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(smem + L::K_OFF + c * 16384, &tm_qkv, kv_full, kcol + c * 64, row0 + k0);
        tma_load_2d(smem + L::V_OFF + c * 16384, &tm_qkv, kv_full, vcol + c * 64, row0 + k0);
      }
      for (int n = 0; n < n_items; ++n) {
        const int s = n % ST;
        const int hq = kvh * group + n / n_i, i = i_start + n % n_i;
        if (!wait_bar(&q_empty[s], ((n / ST) & 1) ^ 1, err, 31)) break;
        // lse and D of this query block ride along (row-vectors of the (B, H, T) layouts)
        const int nq = min(kBN, a.T - i * kBN);
        const uint32_t vbytes = (uint32_t)(((nq + 3) & ~3) * 4);
        bar_arrive_expect_tx(&q_full[s], 2 * L::T_BYTES + 2 * vbytes);
        const int64_t vbase = ((int64_t)b * a.H + hq) * a.T + (int64_t)i * kBN;
        bulk_load(smem + L::VEC_OFF + s * 1024, a.lse + vbase, vbytes, &q_full[s]);
        bulk_load(smem + L::VEC_OFF + s * 1024 + 512, a.dsum + vbase, vbytes, &q_full[s]);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(smem + L::Q_OFF + s * L::T_BYTES + c * 16384, &tm_qkv, &q_full[s], hq * HD + c * 64,
                      row0 + i * kBN);
          tma_load_2d(smem + L::DO_OFF + s * L::T_BYTES + c * 16384, &tm_do, &q_full[s], hq * HD + c * 64,
                      row0 + i * kBN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_bf16(kBM, kBN, false, false);   // S^T, dP^T
      constexpr uint32_t id_kv = make_idesc_bf16(kBM, HD, false, true);   // dV, dK (B MN-major)
      constexpr uint32_t id_q = make_idesc_bf16(kBN, HD, true, true);     // dQ (A = dS MN-major)
      const uint32_t k_addr = smem_u32(smem + L::K_OFF), v_addr = smem_u32(smem + L::V_OFF);
      const uint32_t p_addr = smem_u32(smem + L::P_OFF), ds_addr = smem_u32(smem + L::DS_OFF);
      bool ok = wait_bar(kv_full, 0, err, 32);
      for (int n = 0; n < n_items && ok; ++n) {
        const int s = n % ST;
        if (!wait_bar(&q_full[s], (n / ST) & 1, err, 33)) { ok = false; break; }
        if (!wait_bar(tm_free, (n & 1) ^ 1, err, 34)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + s * L::T_BYTES);
        const uint32_t do_addr = smem_u32(smem + L::DO_OFF + s * L::T_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_f16(tmem + C_S, make_sw128_desc(k_addr + off, 16, 1024), make_sw128_desc(q_addr + off, 16, 1024), id_s,
                  k > 0);
        }
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_f16(tmem + C_DP, make_sw128_desc(v_addr + off, 16, 1024), make_sw128_desc(do_addr + off, 16, 1024), id_s,
                  k > 0);
        }
        mma_commit(s_full);
        if (!wait_bar(pds_full, n & 1, err, 35)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          const uint32_t offk = (k >> 2) * 16384 + (k & 3) * 32;  // K-major step over queries
          const uint32_t offm = k * 2048;                          // MN-major step over queries
          mma_f16(tmem + C_DV, make_sw128_desc(p_addr + offk, 16, 1024), make_sw128_desc(do_addr + offm, 16384, 1024),
                  id_kv, (n > 0 || k > 0) ? 1u : 0u);
          mma_f16(tmem + C_DK, make_sw128_desc(ds_addr + offk, 16, 1024), make_sw128_desc(q_addr + offm, 16384, 1024),
                  id_kv, (n > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&q_empty[s]);  // dQ reads no Q / dO: the stage can refill once dV / dK are done
#pragma unroll
        for (int k = 0; k < kBM / 16; ++k) {  // contraction over keys
          mma_f16(tmem + C_DQ, make_sw128_desc(ds_addr + k * 2048, 16384, 1024),
                  make_sw128_desc(k_addr + k * 2048, 16384, 1024), id_q, k > 0);
        }
        mma_commit(dq_full);
        mma_commit(pds_empty);
      }
      if (ok) mma_commit(dkv_full);
    }
  } else if (warp >= 2) {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // column half handled by this warp (2 warps per lane quadrant)
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int kk = k0 + r;  // this thread's key (S^T / dP^T phase)
    uint8_t* stg = smem + L::STG_OFF + (warp - 2) * (L::EPI_BUFS * 4096);
    int sbuf = 0;
    bool ok = true;
    for (int n = 0; n < n_items; ++n) {
      const int hq = kvh * group + n / n_i, i = i_start + n % n_i;
      const int qbase = i * kBN;
      // s_full implies this item's Q/dO stage (and its -lse log2(e) / -scale D vectors) has landed
      const float* nl_s = reinterpret_cast<const float*>(smem + L::VEC_OFF + (n % ST) * 1024);
      const float* nd_s = nl_s + 128;
      if (!wait_bar(s_full, n & 1, err, 36)) { ok = false; break; }
      if (!wait_bar(pds_empty, (n & 1) ^ 1, err, 37)) { ok = false; break; }
      tc_fence_after();
      uint8_t* pt = smem + L::P_OFF;
      uint8_t* dst = smem + L::DS_OFF;
      const bool diag = a.causal && (qbase < k0 + kBM);
      const bool key_ok = kk < a.T;
      const bool q_tail = qbase + kBN > a.T;  // columns past T hold stale lse / D: mask them
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;
        uint32_t sv[32], dv[32];
        tmem_ld32(tmem + lane_off + C_S + c * 32, sv);
        tmem_ld32(tmem + lane_off + C_DP + c * 32, dv);
        tmem_wait_ld();
        // the same packed form as the pipelined kernel: x = scale log2(e) S - lse log2(e),
        // dS = P (scale dP - scale D) with both addends prepared by the pre-pass
        float p[32], ds[32];
        const bool masked = diag || !key_ok || q_tail;
        const float4* l4 = reinterpret_cast<const float4*>(nl_s + c * 32);
        const float4* d4 = reinterpret_cast<const float4*>(nd_s + c * 32);
        const float2 sl2 = make_float2(a.scale_log2, a.scale_log2), sc2 = make_float2(a.scale, a.scale);
#pragma unroll
        for (int g4 = 0; g4 < 8; ++g4) {
          const float4 lv = l4[g4], dd = d4[g4];
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int e = 4 * g4 + 2 * h2;
            const float2 x = fma2(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sl2,
                                  h2 ? make_float2(lv.z, lv.w) : make_float2(lv.x, lv.y));
            float2 pe;
            if (kBwdPolyEvery > 0 && (e >> 1) % kBwdPolyEvery == kBwdPolyEvery - 1) {
              pe.x = ex2_poly(x.x);
              pe.y = ex2_poly(x.y);
            } else {
              pe.x = ex2_approx(x.x);
              pe.y = ex2_approx(x.y);
            }
            if (masked) {
              const int qi = qbase + c * 32 + e;
              pe.x = (key_ok && (!diag || qi >= kk) && qi < a.T) ? pe.x : 0.f;
              pe.y = (key_ok && (!diag || qi + 1 >= kk) && qi + 1 < a.T) ? pe.y : 0.f;
            }
            const float2 dsv = mul2(pe, fma2(make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), sc2,
                                             h2 ? make_float2(dd.z, dd.w) : make_float2(dd.x, dd.y)));
            p[e] = pe.x;
            p[e + 1] = pe.y;
            ds[e] = dsv.x;
            ds[e + 1] = dsv.y;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          *reinterpret_cast<BF16x8*>(pt + sw_unit(r, c * 4 + u)) = float_to_bf16x8(p + u * 8);
          *reinterpret_cast<BF16x8*>(dst + sw_unit(r, c * 4 + u)) = float_to_bf16x8(ds + u * 8);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      bar_arrive(pds_full);
      // dQ rows (thread = query row of this block): stage as 32x32 fp32 boxes, TMA reduce-add
      if (!wait_bar(dq_full, n & 1, err, 38)) { ok = false; break; }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HD / 64; ++c) {
        const int col = half * (HD / 2) + c * 32;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + C_DQ + col, v);
        if (lane == 0) bulk_wait_read<L::EPI_BUFS - 1>();
        __syncwarp();
        uint8_t* buf = stg + sbuf * 4096;
        sbuf = (sbuf + 1) % L::EPI_BUFS;
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]), __uint_as_float(v[4 * u + 2]),
                          __uint_as_float(v[4 * u + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tm_dq, buf, hq * HD + col, row0 + qbase + quad * 32);
          bulk_commit();
        }
      }
      tc_fence_before();
      bar_arrive(tm_free);
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
    // dK (RoPE backward; dS carried the scale) and dV: the two warps of a lane quadrant each take
    // HD/4 of the HD/2 column pairs (e, e + HD/2) of both, 16 at a time. A quadrant's 32 full rows
    // leave through TMA stores of 32 x 64 bf16 boxes (HD/64 per matrix) staged with the 128B
    // swizzle in the P / dS buffers, which no MMA reads any more; per-thread stores of 16-byte
    // pieces of 32 rows are many times slower. A ragged last key block keeps per-thread stores.
    if (ok && wait_bar(dkv_full, 0, err, 39)) {
      tc_fence_after();
      constexpr int NB = HD / 64;  // boxes per matrix and quadrant
      const bool box = k0 + quad * 32 + 32 <= a.T;  // uniform across the quadrant's two warps
      uint8_t* stg = smem + L::P_OFF + quad * (2 * NB * 4096);  // dK boxes, then dV boxes
      const int64_t grow = (int64_t)(row0 + min(kk, a.T - 1)) * a.ld_qkv;
      const int sw = lane & 7;
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {  // 0: dV, 1: dK
        const uint32_t col = m ? C_DK : C_DV;
        bf16* drow = a.dqkv + grow + (m ? (a.H + kvh) : (a.H + a.KV + kvh)) * HD;
        uint8_t* mst = stg + (m ? 0 : NB * 4096);
#pragma unroll 1
        for (int jj = 0; jj < HD / 64; ++jj) {
          const int e0 = half * (HD / 4) + jj * 16;  // first column of this step's pairs
          uint32_t v1[16], v2[16];
          tmem_ld16(tmem + lane_off + col + e0, v1);
          tmem_ld16(tmem + lane_off + col + HD / 2 + e0, v2);
          tmem_wait_ld();
          float x1[16], x2[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            x1[e] = __uint_as_float(v1[e]);
            x2[e] = __uint_as_float(v2[e]);
          }
          if (m == 1 && kk < a.T) {
            const float4* cr = reinterpret_cast<const float4*>(a.cos_t + (int64_t)kk * HD + e0);
            const float4* sr = reinterpret_cast<const float4*>(a.sin_t + (int64_t)kk * HD + e0);
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              const float4 c1 = cr[e4], c2 = cr[e4 + HD / 8], s1 = sr[e4], s2 = sr[e4 + HD / 8];
              const float cl[4] = {c1.x, c1.y, c1.z, c1.w}, ch[4] = {c2.x, c2.y, c2.z, c2.w};
              const float sl[4] = {s1.x, s1.y, s1.z, s1.w}, sh[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int e = e4 * 4 + q;
                const float a1 = x1[e], a2 = x2[e];
                x1[e] = a1 * cl[q] + a2 * sh[q];
                x2[e] = a2 * ch[q] - a1 * sl[q];
              }
            }
          }
          if (box) {
            // columns e0 .. e0 + 15 and e0 + HD/2 ..: box (c / 64), 16-byte unit (c % 64) / 8
            const int u0 = (e0 % 64) / 8;
            uint8_t* r1 = mst + (e0 / 64) * 4096 + lane * 128;
            uint8_t* r2 = mst + ((e0 + HD / 2) / 64) * 4096 + lane * 128;
            *reinterpret_cast<BF16x8*>(r1 + ((u0 ^ sw) << 4)) = float_to_bf16x8(x1);
            *reinterpret_cast<BF16x8*>(r1 + (((u0 + 1) ^ sw) << 4)) = float_to_bf16x8(x1 + 8);
            *reinterpret_cast<BF16x8*>(r2 + ((u0 ^ sw) << 4)) = float_to_bf16x8(x2);
            *reinterpret_cast<BF16x8*>(r2 + (((u0 + 1) ^ sw) << 4)) = float_to_bf16x8(x2 + 8);
          } else if (kk < a.T) {
            *reinterpret_cast<BF16x8*>(drow + e0) = float_to_bf16x8(x1);
            *reinterpret_cast<BF16x8*>(drow + e0 + 8) = float_to_bf16x8(x1 + 8);
            *reinterpret_cast<BF16x8*>(drow + HD / 2 + e0) = float_to_bf16x8(x2);
            *reinterpret_cast<BF16x8*>(drow + HD / 2 + e0 + 8) = float_to_bf16x8(x2 + 8);
          }
        }
      }
      if (box) {
        fence_proxy_async_smem();
        named_bar_sync(1 + quad, 64);  // both warps' halves of the quadrant's boxes are staged
        if (lane == 0) {
          // the first warp stores the dK boxes, the second the dV boxes
          const int gcol = (half == 0 ? (a.H + kvh) : (a.H + a.KV + kvh)) * HD;
          uint8_t* src = stg + (half == 0 ? 0 : NB * 4096);
#pragma unroll
          for (int bx = 0; bx < NB; ++bx) tma_store_2d(&tm_dkv, src + bx * 4096, gcol + bx * 64, row0 + k0 + quad * 32);
          bulk_commit();
          bulk_wait<0>();  // the boxes are read (and written) before the CTA's shared memory goes away
        }
        __syncwarp();
      }
    }
  }
  pdl_trigger();  // this CTA is done: the next kernel in the stream may be scheduled
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<TMEM_COLS>(tmem);
  }
}

// ---------------------------------------------------------------- pipelined kernel (hd = 64)
// Same math as flash_bwd_kernel, software-pipelined over the query blocks of a CTA so the
// tensor core and the compute warps overlap:
//   MMA warp, step n:  wait P/dS(n) -> S^T, dP^T of block n+1 -> dV, dK += ... (n)
//                      -> wait dQ(n-1) drained -> dQ(n)
//   compute warps:     P, dS of block n (S^T/dP^T(n) already in TMEM) -> drain dQ(n-1)
// so block n+1's S^T/dP^T and block n's dV/dK/dQ run while the compute warps turn block
// n+1 into P/dS. P and dS are double-buffered in shared memory; dQ leaves TMEM one block
// late, staged in the block's P buffer (its dV MMAs are done) and reduced into the fp32 dQ
// accumulator by TMA. TMEM: S^T 0-127, dP^T 128-255, dV 256-319, dK 320-383, dQ 384-447.
struct BwdSmemP {
  static constexpr uint32_t TILE = 128 * 64 * 2;  // one 128 x 64 bf16 tile (16 KB)
  static constexpr uint32_t K_OFF = 0;
  static constexpr uint32_t V_OFF = K_OFF + TILE;
  static constexpr uint32_t Q_OFF = V_OFF + TILE;         // 2 stages
  static constexpr uint32_t DO_OFF = Q_OFF + 2 * TILE;    // 2 stages
  static constexpr uint32_t P_OFF = DO_OFF + 2 * TILE;    // 2 buffers of 128 x 128 bf16
  static constexpr uint32_t DS_OFF = P_OFF + 2 * 32768;   // 2 buffers
  static constexpr uint32_t VEC_OFF = DS_OFF + 2 * 32768; // per stage: lse (128) + D (128) floats
  static constexpr uint32_t BAR_OFF = VEC_OFF + 2 * 1024;
  static constexpr uint32_t TOTAL = BAR_OFF + 256;        // the base must be 1024-aligned (checked)
};
static_assert(BwdSmemP::TOTAL <= 232448, "pipelined attention backward exceeds 227 KB of shared memory");


// Tiles are (kv head, 128-key block) pairs; a persistent CTA per SM walks its share in a
// snake order over rounds (round r: tile r G + i, or r G + G - 1 - i on odd rounds), which
// puts the long causal tiles (low key blocks) first and balances the CTAs' sums. Every
// barrier phase runs on counters that continue across tiles, so one CTA keeps its TMEM,
// barriers and warm caches for all of its tiles, and the MMAs of a tile's first query block
// run while the compute warps finish the previous tile's dK / dV epilogue.
__device__ __forceinline__ int snake_tile(int r, int i, int G) { return r * G + ((r & 1) ? (G - 1 - i) : i); }

// VARIANT 0: the kernel; 2: a timing skeleton with the P / dS arithmetic replaced by copies
// (wrong results; it measures the MMA / TMA / barrier structure alone), chosen at run time with
// LLMT_ATTN_VARIANT for measurements only.
template <int VARIANT>
__global__ void __launch_bounds__(kBwdThreads, 1)
flash_bwd_pipelined_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                           const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dkv,
                           const AttnBwdArgs a) {
  pdl_wait();
  using L = BwdSmemP;
  constexpr int HD = 64;
  constexpr int TMEM_COLS = 512;
  constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // the layout has no slack for realignment
    if (threadIdx.x == 0) atomicCAS(a.err, 0, 40);
    return;
  }
  uint8_t* smem = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;       // [2]
  uint64_t* q_empty = bars + 3;      // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* pds_full = bars + 6;     // 256 arrivals
  uint64_t* pds_empty = bars + 7;    // [2]
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_free = bars + 10;     // 256 arrivals
  uint64_t* dkv_full = bars + 11;
  uint64_t* stage_free = bars + 12;  // 8 arrivals: every compute warp's dQ reduce has read its staging
  uint64_t* kv_empty = bars + 13;    // the tile's MMAs have finished reading K / V
  uint64_t* dkv_free = bars + 14;    // 256 arrivals: the tile's dK / dV are out of TMEM
  uint64_t* st_read = bars + 15;     // 256 arrivals: S^T / dP^T of the block are in registers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int group = a.H / a.KV;
  const int nqb = (int)cdiv(a.T, kBN);
  const int n_bk = a.B * a.KV;
  const int n_tiles = n_bk * nqb;
  const int G = gridDim.x;
  int* err = a.err;

  if (threadIdx.x == 0) {
    bar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      bar_init(&q_full[s], 1);
      bar_init(&q_empty[s], 1);
      bar_init(&pds_empty[s], 1);
    }
    bar_init(s_full, 1);
    bar_init(pds_full, kComputeThreads);
    bar_init(dq_full, 1);
    bar_init(dq_free, kComputeThreads);
    bar_init(dkv_full, 1);
    bar_init(stage_free, 8);
    bar_init(kv_empty, 1);
    bar_init(dkv_free, kComputeThreads);
    bar_init(st_read, kComputeThreads);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // tile t -> (b, kv head, key block); key blocks vary slowest so low (long) ones come first
  struct Tile {
    int b, kvh, kb, i_start, n_i, n_items, row0, k0;
  };
  auto tile_of = [&](int t) {
    Tile x;
    x.kb = t / n_bk;
    const int bk = t % n_bk;
    x.b = bk / a.KV;
    x.kvh = bk % a.KV;
    x.i_start = a.causal ? x.kb : 0;
    x.n_i = nqb - x.i_start;
    x.n_items = group * x.n_i;
    x.row0 = x.b * a.T;
    x.k0 = x.kb * kBM;
    return x;
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv);
      prefetch_tmap(&tm_do);
      int it = 0, tl = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++tl) {
        const int t = snake_tile(r, blockIdx.x, G);
        if (t >= n_tiles) break;
        const Tile x = tile_of(t);
        const int kcol = (a.H + x.kvh) * HD, vcol = (a.H + a.KV + x.kvh) * HD;
        for (int n = 0; n < x.n_items; ++n, ++it) {
          const int s = it & 1;
          const int hq = x.kvh * group + n / x.n_i, i = x.i_start + n % x.n_i;
          if (!wait_bar(&q_empty[s], ((it >> 1) & 1) ^ 1, err, 41)) { ok = false; break; }
          const int nq = min(kBN, a.T - i * kBN);
          const uint32_t vbytes = (uint32_t)(((nq + 3) & ~3) * 4);
          bar_arrive_expect_tx(&q_full[s], 2 * L::TILE + 2 * vbytes);
          const int64_t vbase = ((int64_t)x.b * a.H + hq) * a.T + (int64_t)i * kBN;
          bulk_load(smem + L::VEC_OFF + s * 1024, a.lse + vbase, vbytes, &q_full[s]);
          bulk_load(smem + L::VEC_OFF + s * 1024 + 512, a.dsum + vbase, vbytes, &q_full[s]);
          tma_load_2d(smem + L::Q_OFF + s * L::TILE, &tm_qkv, &q_full[s], hq * HD, x.row0 + i * kBN);
          tma_load_2d(smem + L::DO_OFF + s * L::TILE, &tm_do, &q_full[s], hq * HD, x.row0 + i * kBN);
          if (n == 0) {
            // the tile's first Q / dO are already in flight; K / V wait for the previous tile's MMAs
            if (tl > 0 && !wait_bar(kv_empty, (tl - 1) & 1, err, 53)) { ok = false; break; }
            bar_arrive_expect_tx(kv_full, 2 * L::TILE);
            tma_load_2d(smem + L::K_OFF, &tm_qkv, kv_full, kcol, x.row0 + x.k0);
            tma_load_2d(smem + L::V_OFF, &tm_qkv, kv_full, vcol, x.row0 + x.k0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_bf16(kBM, kBN, false, false);  // S^T, dP^T
      constexpr uint32_t id_kv = make_idesc_bf16(kBM, HD, false, true);  // dV, dK (B MN-major)
      constexpr uint32_t id_q = make_idesc_bf16(kBN, HD, true, true);    // dQ (A = dS MN-major)
      const uint32_t k_addr = smem_u32(smem + L::K_OFF), v_addr = smem_u32(smem + L::V_OFF);
      auto issue_sdp = [&](int s) {
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + s * L::TILE);
        const uint32_t do_addr = smem_u32(smem + L::DO_OFF + s * L::TILE);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          mma_f16(tmem + C_S, make_sw128_desc(k_addr + k * 32, 16, 1024), make_sw128_desc(q_addr + k * 32, 16, 1024),
                  id_s, k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          mma_f16(tmem + C_DP, make_sw128_desc(v_addr + k * 32, 16, 1024), make_sw128_desc(do_addr + k * 32, 16, 1024),
                  id_s, k > 0);
        mma_commit(s_full);
      };
      int it = 0, tl = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++tl) {
        const int t = snake_tile(r, blockIdx.x, G);
        if (t >= n_tiles) break;
        const Tile x = tile_of(t);
        if (!wait_bar(kv_full, tl & 1, err, 42)) break;
        if (!wait_bar(&q_full[it & 1], (it >> 1) & 1, err, 43)) break;
        tc_fence_after();
        issue_sdp(it & 1);
        for (int n = 0; n < x.n_items; ++n) {
          const int g = it + n;
          const int s = g & 1, pb = g & 1;
          // the next block's S^T / dP^T as soon as this block's are in the compute warps'
          // registers, so those MMAs run under this block's softmax
          if (n + 1 < x.n_items) {
            if (!wait_bar(st_read, g & 1, err, 55)) { ok = false; break; }
            if (!wait_bar(&q_full[(g + 1) & 1], ((g + 1) >> 1) & 1, err, 45)) { ok = false; break; }
            tc_fence_after();
            issue_sdp((g + 1) & 1);
          }
          if (!wait_bar(pds_full, g & 1, err, 44)) { ok = false; break; }
          tc_fence_after();
          // the previous tile's dK / dV must be out of TMEM before they are overwritten
          if (n == 0 && tl > 0 && !wait_bar(dkv_free, (tl - 1) & 1, err, 54)) { ok = false; break; }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + L::Q_OFF + s * L::TILE);
          const uint32_t do_addr = smem_u32(smem + L::DO_OFF + s * L::TILE);
          const uint32_t p_addr = smem_u32(smem + L::P_OFF + pb * 32768);
          const uint32_t ds_addr = smem_u32(smem + L::DS_OFF + pb * 32768);
#pragma unroll
          for (int k = 0; k < kBN / 16; ++k) {
            const uint32_t offk = (k >> 2) * 16384 + (k & 3) * 32;  // K-major step over queries
            const uint32_t offm = k * 2048;                          // MN-major step over queries
            mma_f16(tmem + C_DV, make_sw128_desc(p_addr + offk, 16, 1024),
                    make_sw128_desc(do_addr + offm, 16384, 1024), id_kv, (n > 0 || k > 0) ? 1u : 0u);
            mma_f16(tmem + C_DK, make_sw128_desc(ds_addr + offk, 16, 1024),
                    make_sw128_desc(q_addr + offm, 16384, 1024), id_kv, (n > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&q_empty[s]);  // dQ reads no Q / dO: the stage can refill as soon as dV / dK are done
          if (g > 0 && !wait_bar(dq_free, (g - 1) & 1, err, 46)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < kBM / 16; ++k)  // contraction over keys
            mma_f16(tmem + C_DQ, make_sw128_desc(ds_addr + k * 2048, 16384, 1024),
                    make_sw128_desc(k_addr + k * 2048, 16384, 1024), id_q, k > 0);
          mma_commit(dq_full);
          mma_commit(&pds_empty[pb]);
        }
        if (!ok) break;
        mma_commit(dkv_full);  // this tile's dK / dV are final
        mma_commit(kv_empty);  // and its K / V are no longer read
        it += x.n_items;
      }
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // column half handled by this warp (2 warps per lane quadrant)
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    bool epi_pending = false;  // this warp's last dK / dV TMA store may still be reading its staging
    int it = 0, tl = 0;
    for (int rr = 0; ok; ++rr, ++tl) {
      const int t = snake_tile(rr, blockIdx.x, G);
      if (t >= n_tiles) break;
      const Tile x = tile_of(t);
      const int kk = x.k0 + r;  // this thread's key (S^T / dP^T phase)
      // dQ of item n of this tile: TMEM -> registers, staged as one 32 x 32 fp32 box per
      // warp (SW128) in the item's P buffer (its MMAs are done) -> TMA reduce-add into dq_acc
      auto drain_dq = [&](int n) -> bool {
        const int g = it + n;
        if (!wait_bar(dq_full, g & 1, err, 47)) return false;
        tc_fence_after();
        const int hq = x.kvh * group + n / x.n_i, qb = (x.i_start + n % x.n_i) * kBN;
        const int col = half * 32;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + C_DQ + col, v);
        tmem_wait_ld();
        tc_fence_before();
        bar_arrive(dq_free);
        uint8_t* buf = smem + L::P_OFF + (g & 1) * 32768 + (warp - 2) * 4096;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]), __uint_as_float(v[4 * u + 2]),
                          __uint_as_float(v[4 * u + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // rows past T (a ragged last block) carry zeros: their dS was masked
          tma_reduce_add_2d(&tm_dq, buf, hq * HD + col, x.row0 + qb + quad * 32);
          bulk_commit();
        }
        return true;
      };
      for (int n = 0; n < x.n_items && ok; ++n) {
        const int g = it + n;
        const int pb = g & 1;
        const int i = x.i_start + n % x.n_i;
        const int qbase = i * kBN;
        const float* nl_s = reinterpret_cast<const float*>(smem + L::VEC_OFF + (g & 1) * 1024);  // -lse log2(e)
        const float* nd_s = nl_s + 128;                                                           // -scale D
        if (!wait_bar(s_full, g & 1, err, 48)) { ok = false; break; }
        if (!wait_bar(&pds_empty[pb], ((g >> 1) & 1) ^ 1, err, 49)) { ok = false; break; }
        if (g >= 2) {
          // buffer pb staged dQ(g - 2) for every warp's TMA reduce (issued at the end of the
          // previous block, this warp's latest bulk group): all of them must have read it.
          if (lane == 0) {
            bulk_wait_read<0>();
            bar_arrive(stage_free);
          }
          epi_pending = false;
          __syncwarp();
          if (!wait_bar(stage_free, (g - 2) & 1, err, 52)) { ok = false; break; }
        }
        tc_fence_after();
        uint8_t* pt = smem + L::P_OFF + pb * 32768;
        uint8_t* dst = smem + L::DS_OFF + pb * 32768;
        // valid queries of this key row: [q_lo, q_hi) of the block (causal: query >= key; query < T;
        // none for keys past T). One predicated loop serves the masked and the full blocks, which
        // keeps the code small: the first block of every tile is masked.
        const bool key_ok = kk < a.T;
        const int q_lo = (a.causal && qbase < x.k0 + kBM) ? kk - qbase : 0;
        const int q_hi = key_ok ? min(kBN, a.T - qbase) : 0;
        // this warp's 64 columns of S^T and dP^T, 32 at a time; after the second chunk is in
        // registers the columns are released, so the next block's S^T / dP^T MMAs can start.
        // Per pair of queries: x = scale log2(e) S - lse log2(e) (one packed FMA, the lse term
        // negated and scaled by the pre-pass), P = 2^x (one pair in kBwdPolyEvery on the FMA
        // pipe), dS = P (scale dP - scale D) (a packed FMA and a packed multiply): dS carries the
        // softmax scale, so dK and dQ need no scaling. Blocks with no masked query in this key row
        // (all but the diagonal block, and keys past T) skip the mask.
        auto chunk = [&](int cc, auto masked_tag) {
          constexpr bool MASKED = decltype(masked_tag)::value;
          const int c = half * 2 + cc;
          uint32_t sv[32], dv[32];
          tmem_ld32(tmem + lane_off + C_S + c * 32, sv);
          tmem_ld32(tmem + lane_off + C_DP + c * 32, dv);
          tmem_wait_ld();
          if (cc == 1) {
            tc_fence_before();
            bar_arrive(st_read);
          }
          const int lo = q_lo - c * 32, hi = q_hi - c * 32;
          const float4* l4 = reinterpret_cast<const float4*>(nl_s + c * 32);
          const float4* d4 = reinterpret_cast<const float4*>(nd_s + c * 32);
          const float2 sl2 = make_float2(a.scale_log2, a.scale_log2), sc2 = make_float2(a.scale, a.scale);
          float p[32], ds[32];
#pragma unroll
          for (int g4 = 0; g4 < 8; ++g4) {
            const float4 lv = l4[g4], dd = d4[g4];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int e = 4 * g4 + 2 * h2;
              const float2 s2 = make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
              const float2 d2 = make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1]));
              if (VARIANT == 2) {
                p[e] = s2.x;
                p[e + 1] = s2.y;
                ds[e] = d2.x;
                ds[e + 1] = d2.y;
                continue;
              }
              const float2 x = fma2(s2, sl2, h2 ? make_float2(lv.z, lv.w) : make_float2(lv.x, lv.y));
              float2 pe;
              if (kBwdPolyEvery > 0 && (e >> 1) % kBwdPolyEvery == kBwdPolyEvery - 1) {
                pe.x = ex2_poly(x.x);
                pe.y = ex2_poly(x.y);
              } else {
                pe.x = ex2_approx(x.x);
                pe.y = ex2_approx(x.y);
              }
              if (MASKED) {
                pe.x = (e >= lo && e < hi) ? pe.x : 0.f;
                pe.y = (e + 1 >= lo && e + 1 < hi) ? pe.y : 0.f;
              }
              const float2 dsv = mul2(pe, fma2(d2, sc2, h2 ? make_float2(dd.z, dd.w) : make_float2(dd.x, dd.y)));
              p[e] = pe.x;
              p[e + 1] = pe.y;
              ds[e] = dsv.x;
              ds[e + 1] = dsv.y;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            *reinterpret_cast<BF16x8*>(pt + sw_unit(r, c * 4 + u)) = float_to_bf16x8(p + u * 8);
            *reinterpret_cast<BF16x8*>(dst + sw_unit(r, c * 4 + u)) = float_to_bf16x8(ds + u * 8);
          }
        };
        // warp-uniform choice: tcgen05.ld is a warp-collective instruction, so the whole warp
        // takes one path (the diagonal block's first key row alone would need no mask)
        if (__all_sync(0xffffffffu, q_lo <= 0 && q_hi >= kBN)) {
          chunk(0, std::false_type{});
          chunk(1, std::false_type{});
        } else {
          chunk(0, std::true_type{});
          chunk(1, std::true_type{});
        }
        tc_fence_before();
        fence_proxy_async_smem();
        bar_arrive(pds_full);
        if (n > 0 && !drain_dq(n - 1)) { ok = false; break; }
      }
      // The RoPE table slices of this warp's dK column pairs (16 * half + [0, 16) and + 32): cos
      // loaded before the last dQ drain, sin after it, so that their latency passes under the
      // drain and the dK / dV wait (both before would spill).
      float4 pc[8], ps[8];
      const int64_t toff = (int64_t)min(kk, a.T - 1) * HD + half * 16;
#pragma unroll
      for (int e4 = 0; e4 < 4; ++e4) {
        pc[e4] = ld_f4(a.cos_t + toff + 4 * e4);
        pc[4 + e4] = ld_f4(a.cos_t + toff + 32 + 4 * e4);
      }
      if (ok && x.n_items > 0) ok = drain_dq(x.n_items - 1);
#pragma unroll
      for (int e4 = 0; e4 < 4; ++e4) {
        ps[e4] = ld_f4(a.sin_t + toff + 4 * e4);
        ps[4 + e4] = ld_f4(a.sin_t + toff + 32 + 4 * e4);
      }
      // dK (RoPE backward; dS carried the scale) by the first warp of each quadrant, dV by the
      // second; column pairs (e, e + 32) are handled 16 at a time to keep registers low
      // dK (RoPE backward; dS carried the scale) and dV: the two warps of a lane quadrant each take
      // 16 of the 32 column pairs (e, e + 32) of both. A quadrant's 32 full rows leave through one
      // TMA store per matrix of a 32 x 64 bf16 box staged (128B swizzle) in dS^T buffer 0, which no
      // MMA reads any more: per-thread stores, each a 16-byte piece of 32 different rows, took about
      // 25 times as long. A ragged last key block keeps per-thread stores (its rows past T would
      // fall into the next sequence).
      if (ok && wait_bar(dkv_full, tl & 1, err, 50)) {
        tc_fence_after();
        const bool box = x.k0 + quad * 32 + 32 <= a.T;  // uniform across the quadrant's two warps
        uint8_t* stg_k = smem + L::DS_OFF + quad * 8192;
        uint8_t* stg_v = stg_k + 4096;
        if (box && epi_pending) {  // the quadrant's previous TMA stores must have read the boxes
          if (lane == 0) bulk_wait_read<0>();
          named_bar_sync(1 + quad, 64);
        }
        const int64_t grow = (int64_t)(x.row0 + min(kk, a.T - 1)) * a.ld_qkv;
        bf16* krow = a.dqkv + grow + (a.H + x.kvh) * HD;
        bf16* vrow = a.dqkv + grow + (a.H + a.KV + x.kvh) * HD;
        const int sw = lane & 7;
        // columns 16 * half + [0, 16) -> 16-byte units 2 half, 2 half + 1; + 32 -> units 4 + 2 half, 5 + 2 half
        auto put = [&](uint8_t* stg, bf16* grow_ptr, const float* x1, const float* x2) {
          if (box) {
            uint8_t* row = stg + lane * 128;
            *reinterpret_cast<BF16x8*>(row + (((2 * half) ^ sw) << 4)) = float_to_bf16x8(x1);
            *reinterpret_cast<BF16x8*>(row + (((2 * half + 1) ^ sw) << 4)) = float_to_bf16x8(x1 + 8);
            *reinterpret_cast<BF16x8*>(row + (((4 + 2 * half) ^ sw) << 4)) = float_to_bf16x8(x2);
            *reinterpret_cast<BF16x8*>(row + (((5 + 2 * half) ^ sw) << 4)) = float_to_bf16x8(x2 + 8);
          } else if (kk < a.T) {
            *reinterpret_cast<BF16x8*>(grow_ptr + half * 16) = float_to_bf16x8(x1);
            *reinterpret_cast<BF16x8*>(grow_ptr + half * 16 + 8) = float_to_bf16x8(x1 + 8);
            *reinterpret_cast<BF16x8*>(grow_ptr + 32 + half * 16) = float_to_bf16x8(x2);
            *reinterpret_cast<BF16x8*>(grow_ptr + 32 + half * 16 + 8) = float_to_bf16x8(x2 + 8);
          }
        };
        {
          uint32_t v1[16], v2[16];
          tmem_ld16(tmem + lane_off + C_DV + half * 16, v1);
          tmem_ld16(tmem + lane_off + C_DV + 32 + half * 16, v2);
          tmem_wait_ld();
          float x1[16], x2[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            x1[e] = __uint_as_float(v1[e]);
            x2[e] = __uint_as_float(v2[e]);
          }
          put(stg_v, vrow, x1, x2);
        }
        {
          uint32_t v1[16], v2[16];
          tmem_ld16(tmem + lane_off + C_DK + half * 16, v1);
          tmem_ld16(tmem + lane_off + C_DK + 32 + half * 16, v2);
          tmem_wait_ld();
          tc_fence_before();
          bar_arrive(dkv_free);  // the next tile's dV / dK may overwrite these columns now
          float x1[16], x2[16];
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const float cl[4] = {pc[e4].x, pc[e4].y, pc[e4].z, pc[e4].w};
            const float ch[4] = {pc[4 + e4].x, pc[4 + e4].y, pc[4 + e4].z, pc[4 + e4].w};
            const float sl[4] = {ps[e4].x, ps[e4].y, ps[e4].z, ps[e4].w};
            const float sh[4] = {ps[4 + e4].x, ps[4 + e4].y, ps[4 + e4].z, ps[4 + e4].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e = e4 * 4 + q;
              const float a1 = __uint_as_float(v1[e]), a2 = __uint_as_float(v2[e]);
              x1[e] = a1 * cl[q] + a2 * sh[q];
              x2[e] = a2 * ch[q] - a1 * sl[q];
            }
          }
          put(stg_k, krow, x1, x2);
        }
        if (box) {
          fence_proxy_async_smem();
          named_bar_sync(1 + quad, 64);  // both halves of both boxes are staged
          if (lane == 0) {
            const int gcol = (half == 0 ? (a.H + x.kvh) : (a.H + a.KV + x.kvh)) * HD;
            tma_store_2d(&tm_dkv, half == 0 ? stg_k : stg_v, gcol, x.row0 + x.k0 + quad * 32);
            bulk_commit();
          }
          epi_pending = true;
        }
      } else {
        ok = false;
      }
      it += x.n_items;
    }
    if (lane == 0) bulk_wait<0>();  // this warp's dQ reductions are complete before exit
    __syncwarp();
  }
  pdl_trigger();  // this CTA is done: the next kernel in the stream may be scheduled
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<TMEM_COLS>(tmem);
  }
}

// D = rowsum(dO * O) per (b, h, t); also zeroes the fp32 dQ accumulator row slice.
// One thread per 8-wide chunk; the HD/8 threads of a (row, head) reduce with shuffles.
// With nlse2 set (both backward kernels) it writes -D * dscale and -lse * log2(e) instead, the two
// addends of their packed FMAs (dS = P (scale dP - scale D), P = 2^(scale log2e S - lse log2e)).
template <int HD>
__global__ void attn_bwd_pre_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dO, float* __restrict__ dsum,
                                    float* __restrict__ dq_acc, int BT, int T, int H, const float* __restrict__ lse,
                                    float* __restrict__ nlse2, float dscale) {
  pdl_wait();
  constexpr int G = HD / 8;  // threads per (row, head): 8 or 16, divides the warp
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)BT * H * G;
  const bool valid = idx < total;
  const int64_t rh = valid ? idx / G : 0;
  const int c = (int)(idx % G) * 8;
  float acc = 0.f;
  if (valid) {
    const int64_t off = rh * HD + c;  // (row, head) pairs are contiguous HD-element slices
    float x[8], y[8];
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(o + off), x);
    bf16x8_to_float(*reinterpret_cast<const BF16x8*>(dO + off), y);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += x[e] * y[e];
    st_f4(dq_acc + off, make_float4(0.f, 0.f, 0.f, 0.f));
    st_f4(dq_acc + off + 4, make_float4(0.f, 0.f, 0.f, 0.f));
  }
#pragma unroll
  for (int w = G / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
  if (valid && c == 0) {
    const int64_t row = rh / H;
    const int h = (int)(rh % H);
    const int b = (int)(row / T), t = (int)(row % T);
    const int64_t i = ((int64_t)b * H + h) * T + t;
    if (nlse2) {
      dsum[i] = -acc * dscale;
      nlse2[i] = -lse[i] * kLog2e;
    } else {
      dsum[i] = acc;
    }
  }
}

// dq (bf16, RoPE backward) <- dq_acc (fp32), into the q columns of the packed dqkv rows.
template <int HD>
__global__ void attn_bwd_post_kernel(const float* __restrict__ dq_acc, bf16* __restrict__ dqkv,
                                     const float* __restrict__ cos_t, const float* __restrict__ sin_t, int BT, int T,
                                     int H, int ld_qkv) {
  pdl_wait();
  constexpr int HALF = HD / 2;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // (row, head, 8-chunk of half)
  constexpr int CH = HALF / 8;
  if (idx >= (int64_t)BT * H * CH) return;
  const int c = (int)(idx % CH) * 8;
  const int64_t rest = idx / CH;
  const int h = (int)(rest % H);
  const int64_t row = rest / H;
  const int t = (int)(row % T);
  const float* src = dq_acc + row * (int64_t)H * HD + h * HD;
  float x1[8], x2[8], y1[8], y2[8];
  float4 a0 = ld_f4(src + c), a1 = ld_f4(src + c + 4), b0 = ld_f4(src + HALF + c), b1 = ld_f4(src + HALF + c + 4);
  x1[0] = a0.x; x1[1] = a0.y; x1[2] = a0.z; x1[3] = a0.w; x1[4] = a1.x; x1[5] = a1.y; x1[6] = a1.z; x1[7] = a1.w;
  x2[0] = b0.x; x2[1] = b0.y; x2[2] = b0.z; x2[3] = b0.w; x2[4] = b1.x; x2[5] = b1.y; x2[6] = b1.z; x2[7] = b1.w;
  const float* cr = cos_t + (int64_t)t * HD;
  const float* sr = sin_t + (int64_t)t * HD;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    y1[e] = x1[e] * cr[c + e] + x2[e] * sr[HALF + c + e];
    y2[e] = x2[e] * cr[HALF + c + e] - x1[e] * sr[c + e];
  }
  bf16* dst = dqkv + row * (int64_t)ld_qkv + h * HD;
  *reinterpret_cast<BF16x8*>(dst + c) = float_to_bf16x8(y1);
  *reinterpret_cast<BF16x8*>(dst + HALF + c) = float_to_bf16x8(y2);
}

template <int HD>
cudaError_t launch_bwd(const CUtensorMap& tq, const CUtensorMap& tdo, const CUtensorMap& tdq, const CUtensorMap& tdkv,
                       const AttnBwdArgs& args, cudaStream_t st) {
  auto kern = flash_bwd_kernel<HD>;
  constexpr size_t smem = BwdSmem<HD>::TOTAL;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  dim3 grid((unsigned)(args.B * args.KV), (unsigned)cdiv(args.T, kBM));
  launch_pdl(kern, grid, kBwdThreads, smem, st, tq, tdo, tdq, tdkv, args);
  return cudaGetLastError();
}

template <int VARIANT>
cudaError_t launch_bwd_pipelined_v(const CUtensorMap& tq, const CUtensorMap& tdo, const CUtensorMap& tdq,
                                   const CUtensorMap& tdkv, const AttnBwdArgs& args, cudaStream_t st) {
  constexpr size_t smem = BwdSmemP::TOTAL;
  auto kern = flash_bwd_pipelined_kernel<VARIANT>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = args.B * args.KV * (int)cdiv(args.T, kBM);
  launch_pdl(kern, std::min(tiles, persistent_sms()), kBwdThreads, smem, st, tq, tdo, tdq, tdkv, args);
  return cudaGetLastError();
}

cudaError_t launch_bwd_pipelined(const CUtensorMap& tq, const CUtensorMap& tdo, const CUtensorMap& tdq,
                                 const CUtensorMap& tdkv, const AttnBwdArgs& args, cudaStream_t st) {
  static const int variant = [] {
    const char* e = getenv("LLMT_ATTN_VARIANT");
    return e ? atoi(e) : 0;
  }();
  return variant == 2 ? launch_bwd_pipelined_v<2>(tq, tdo, tdq, tdkv, args, st)
                      : launch_bwd_pipelined_v<0>(tq, tdo, tdq, tdkv, args, st);
}

}  // namespace

// dqkv (B*T, ld_qkv) bf16 receives the gradient w.r.t. the packed *pre-RoPE* qkv rows.
// dsum (2*B*H*T floats) and dq_acc (B*T*H*hd floats) are caller-provided scratch.
cudaError_t flash_attn_bwd(const void* dO, const void* qkv, int64_t ld_qkv, const void* o, const float* lse,
                           const float* cos_t, const float* sin_t, void* dqkv, float* dsum, float* dq_acc, int B,
                           int T, int H, int KV, int hd, bool causal, float scale, cudaStream_t st) {
  LLMT_REQUIRE(hd == 64 || hd == 128, "flash_attn_bwd: head dim must be 64 or 128");
  LLMT_REQUIRE(KV > 0 && H % KV == 0, "flash_attn_bwd: H must be a multiple of KV");
  LLMT_REQUIRE(tma_ok(qkv, ld_qkv, 2) && tma_ok(dO, (int64_t)H * hd, 2), "flash_attn_bwd: TMA alignment");
  LLMT_REQUIRE(T % 4 == 0 && (reinterpret_cast<uintptr_t>(lse) & 15) == 0,
               "flash_attn_bwd: T must be a multiple of 4 (16-byte lse rows)");
  if (B == 0 || T == 0) return cudaSuccess;
  const int64_t rows = (int64_t)B * T;
  {
    const int64_t n = rows * H * (hd / 8);
    auto k = hd == 64 ? attn_bwd_pre_kernel<64> : attn_bwd_pre_kernel<128>;
    float* nlse2 = dsum + rows * H;
    launch_pdl(k, (unsigned)cdiv(n, 256), 256, 0, st, static_cast<const bf16*>(o), static_cast<const bf16*>(dO), dsum,
               dq_acc, (int)rows, T, H, lse, nlse2, scale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  AttnBwdArgs args{};
  args.lse = dsum + rows * H;  // -lse log2(e); args.dsum holds -scale D (see the pre-pass)
  args.dsum = dsum;
  args.dq_acc = dq_acc;
  args.dqkv = static_cast<bf16*>(dqkv);
  args.cos_t = cos_t;
  args.sin_t = sin_t;
  args.B = B;
  args.T = T;
  args.H = H;
  args.KV = KV;
  args.ld_qkv = (int)ld_qkv;
  args.ld_dq = H * hd;
  args.scale = scale;
  args.scale_log2 = scale * 1.4426950408889634f;
  args.causal = causal ? 1 : 0;
  args.err = attn_err_word();
  alignas(64) CUtensorMap tq, tdo, tdq;
  const bool ok =
      make_tmap_2d(&tq, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)(H + 2 * KV) * hd, rows, ld_qkv, 64, 128) &&
      make_tmap_2d(&tdo, dO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * hd, rows, (uint64_t)H * hd, 64, 128) &&
      make_tmap_2d(&tdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)H * hd, rows, (uint64_t)H * hd, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  LLMT_REQUIRE(ok, "flash_attn_bwd: tensor map rejected");
  // dK / dV boxes of 32 key rows x 64 columns for the TMA-store epilogues
  alignas(64) CUtensorMap tdkv;
  LLMT_REQUIRE(tma_ok(dqkv, ld_qkv, 2) &&
                   make_tmap_2d(&tdkv, dqkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)(H + 2 * KV) * hd, rows,
                                ld_qkv, 64, 32),
               "flash_attn_bwd: dqkv tensor map rejected");
  cudaError_t e = hd == 64 ? launch_bwd_pipelined(tq, tdo, tdq, tdkv, args, st)
                           : launch_bwd<128>(tq, tdo, tdq, tdkv, args, st);
  if (e != cudaSuccess) return e;
  {
    const int64_t n = rows * H * (hd / 16);
    auto k = hd == 64 ? attn_bwd_post_kernel<64> : attn_bwd_post_kernel<128>;
    launch_pdl(k, (unsigned)cdiv(n, 256), 256, 0, st, dq_acc, static_cast<bf16*>(dqkv), cos_t, sin_t, (int)rows, T, H,
                                              (int)ld_qkv);
  }
  return cudaGetLastError();
}

}  // namespace llmt

// Causal flash attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's F.scaled_dot_product_attention(is_causal=True) (bench_train.py:141-142)
// and its output transpose copy (bench_train.py:149): q, k, v are read by TMA straight from the
// packed post-RoPE qkv rows (B*T, (H + 2*KV) * hd) and o is written as (B*T, H*hd), the layout
// the wo GEMM consumes. Online softmax (Milakov & Gimelshein 2018; FlashAttention, Dao et al.).
//
// Persistent: two CTAs per SM (so one CTA's softmax overlaps the other's MMAs) walk the
// (batch*head, 128-query block) tiles, heaviest causal blocks first, in a snake order:
//   warp 0     TMA producer: each tile's Q (double-buffered at head dim 64, so the next tile's
//              Q lands during this one), K/V blocks of 128 keys through a STAGES-deep ring
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S_j  = Q K_j^T   (SS form, M=128, N=128, K=hd)    -> TMEM cols [0, 128)
//                O'_j = P_j V_j   (TS form: P_j read from TMEM)    -> TMEM cols [128, 128+hd)
//   warps 2-5  one thread per query row: row max of S_j (tree reduction, diagonal block
//              masked branch-free), P = 2^(S*scale*log2e - m) on the SFU, row sum, P packed to
//              bf16 and stored back over the consumed S columns with tcgen05.st; O is kept in
//              registers, O = O * 2^(m_old - m_new) + O'_j.
// GQA: query head h reads key/value head h / (H / KV). Keys past T or past the query
// (causal) are masked. Saves lse (B, H, T) in natural-log units for the backward.
#include "../common/common.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.h"

namespace llmt {
int* attn_err_word();
namespace {

using namespace sm100;

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kAttnThreads = 192;

struct AttnFwdArgs {
  bf16* o;
  float* lse;
  int B, T, H, KV, ld_o;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int* err;
};

__device__ int g_attn_err = 0;

template <int HD>
struct FwdSmem {
  static constexpr int STAGES = HD == 64 ? 2 : 1;
  static constexpr int QST = HD == 64 ? 2 : 1;  // Q buffers: the next tile's Q loads during this one
  static constexpr uint32_t Q_BYTES = kBlockM * HD * 2;
  static constexpr uint32_t KV_BYTES = kBlockN * HD * 2;
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = Q_OFF + QST * Q_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + STAGES * KV_BYTES;
  static constexpr uint32_t BAR_OFF = V_OFF + STAGES * KV_BYTES;
  static constexpr uint32_t TOTAL = BAR_OFF + 128 + 1024;
};

// Tiles are (batch x head, 128-query block) pairs; a persistent CTA (two per SM) walks its share in
// a snake order over rounds, query blocks with the most key blocks first. Every barrier phase runs on
// counters that continue across tiles, so TMEM, barriers and the K/V ring persist, and the next
// tile's Q (double-buffered at hd 64) loads while this tile runs.
__device__ __forceinline__ int fwd_snake(int r, int i, int G) { return r * G + ((r & 1) ? (G - 1 - i) : i); }

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 2)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnFwdArgs a) {
  pdl_wait();
  using L = FwdSmem<HD>;
  constexpr int ST = L::STAGES;
  constexpr int QST = L::QST;
  constexpr int TMEM_COLS = 256;        // S/P at [0, 128), O' at [128, 128 + HD)
  constexpr uint32_t C_O = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* k_full = bars + 0;       // [ST]
  uint64_t* v_full = bars + 2;       // [ST]
  uint64_t* kv_empty = bars + 4;     // [ST]
  uint64_t* s_full = bars + 6;
  uint64_t* p_full = bars + 7;       // 128 arrivals
  uint64_t* o_full = bars + 8;
  uint64_t* q_full = bars + 9;       // [QST]
  uint64_t* q_empty = bars + 11;     // [QST]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_bh = a.B * a.H;
  const int nqb = (int)cdiv(a.T, kBlockM);
  const int n_tiles = n_bh * nqb;
  const int G = gridDim.x;
  int* err = a.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&v_full[s], 1);
      bar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < QST; ++s) {
      bar_init(&q_full[s], 1);
      bar_init(&q_empty[s], 1);
    }
    bar_init(s_full, 1);
    bar_init(p_full, 128);
    bar_init(o_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  struct Tile {
    int b, h, q0, kvh, nkv, row0;
  };
  auto tile_of = [&](int t) {
    Tile x;
    const int qb = nqb - 1 - t / n_bh;  // most key blocks first
    const int bh = t % n_bh;
    x.b = bh / a.H;
    x.h = bh % a.H;
    x.q0 = qb * kBlockM;
    x.kvh = x.h / (a.H / a.KV);
    x.nkv = a.causal ? min(qb + 1, (int)cdiv(a.T, kBlockN)) : (int)cdiv(a.T, kBlockN);
    x.row0 = x.b * a.T;  // first packed row of this sequence
    return x;
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv);
      int jj = 0, tl = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++tl) {
        const int t = fwd_snake(r, blockIdx.x, G);
        if (t >= n_tiles) break;
        const Tile x = tile_of(t);
        const int qs = tl % QST;
        if (!wait_bar(&q_empty[qs], ((tl / QST) & 1) ^ 1, err, 10)) break;
        const int qcol = x.h * HD, kcol = (a.H + x.kvh) * HD, vcol = (a.H + a.KV + x.kvh) * HD;
        bar_arrive_expect_tx(&q_full[qs], L::Q_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(smem + L::Q_OFF + qs * L::Q_BYTES + c * 16384, &tm_qkv, &q_full[qs], qcol + c * 64,
                      x.row0 + x.q0);
        for (int j = 0; j < x.nkv; ++j, ++jj) {
          const int s = jj % ST;
          if (!wait_bar(&kv_empty[s], ((jj / ST) & 1) ^ 1, err, 11)) { ok = false; break; }
          bar_arrive_expect_tx(&k_full[s], L::KV_BYTES);
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + L::K_OFF + s * L::KV_BYTES + c * 16384, &tm_qkv, &k_full[s], kcol + c * 64,
                        x.row0 + j * kBlockN);
          bar_arrive_expect_tx(&v_full[s], L::KV_BYTES);
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + L::V_OFF + s * L::KV_BYTES + c * 16384, &tm_qkv, &v_full[s], vcol + c * 64,
                        x.row0 + j * kBlockN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBlockM, HD, false, true);
      int jj = 0, tl = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++tl) {
        const int t = fwd_snake(r, blockIdx.x, G);
        if (t >= n_tiles) break;
        const Tile x = tile_of(t);
        const int qs = tl % QST;
        if (!wait_bar(&q_full[qs], (tl / QST) & 1, err, 12)) break;
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + qs * L::Q_BYTES);
        for (int j = 0; j < x.nkv; ++j, ++jj) {
          const int s = jj % ST;
          if (!wait_bar(&k_full[s], (jj / ST) & 1, err, 16)) { ok = false; break; }
          // P_{jj-1} (aliasing S) must have been read by PV_{jj-1} before S_jj overwrites it.
          if (jj > 0 && !wait_bar(o_full, (jj - 1) & 1, err, 17)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + L::K_OFF + s * L::KV_BYTES);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
            mma_f16(tmem, make_sw128_desc(q_addr + off, 16, 1024), make_sw128_desc(k_addr + off, 16, 1024), idesc_s,
                    k > 0 ? 1u : 0u);
          }
          mma_commit(s_full);
          if (j == x.nkv - 1) mma_commit(&q_empty[qs]);  // the tile's last S has read its Q
          if (!wait_bar(&v_full[s], (jj / ST) & 1, err, 13)) { ok = false; break; }
          if (!wait_bar(p_full, jj & 1, err, 14)) { ok = false; break; }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + L::V_OFF + s * L::KV_BYTES);
#pragma unroll
          for (int k = 0; k < kBlockN / 16; ++k)
            mma_f16_ts(tmem + C_O, tmem + k * 8, make_sw128_desc(v_addr + k * 2048, 16384, 1024), idesc_o,
                       k > 0 ? 1u : 0u);
          mma_commit(o_full);
          mma_commit(&kv_empty[s]);
        }
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the block
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_off;
    const float sl2 = a.scale_log2;
    int jj = 0;
    bool ok = true;
    for (int rr = 0; ok; ++rr) {
      const int t = fwd_snake(rr, blockIdx.x, G);
      if (t >= n_tiles) break;
      const Tile x = tile_of(t);
      const int q = x.q0 + r;
      const int q0 = x.q0;
      float o_acc[HD];
#pragma unroll
      for (int i = 0; i < HD; ++i) o_acc[i] = 0.f;
      float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
      for (int j = 0; j < x.nkv && ok; ++j, ++jj) {
        if (!wait_bar(s_full, jj & 1, err, 19)) { ok = false; break; }
        tc_fence_after();
        const int k0 = j * kBlockN;
        // keys allowed for this row: key < lim (causal: key <= q; always key < T)
        const int lim = a.causal ? min(q + 1, a.T) : a.T;
        const bool need_mask = k0 + kBlockN > (a.causal ? q0 + 1 : a.T) || k0 + kBlockN > a.T;
        // pass 1: row max, 8 independent chains
        float mx8[8];
  #pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
  #pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(t_s + c * 32, v);
          tmem_wait_ld();
          if (need_mask) {
  #pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = (k0 + c * 32 + e < lim) ? __uint_as_float(v[e]) : -INFINITY;
              mx8[e & 7] = fmaxf(mx8[e & 7], x);
            }
          } else {
  #pragma unroll
            for (int e = 0; e < 32; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(v[e]));
          }
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m, mx * sl2);
        const float msub = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = ex2_approx(m - msub);  // m = -inf on the first block -> 0
        // O'_{j-1} finished before S_j started (same MMA issue order), fold it in now.
        if (j > 0) {
          if (!wait_bar(o_full, (jj - 1) & 1, err, 18)) { ok = false; break; }
          tc_fence_after();
  #pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(t_s + C_O + c * 32, v);
            tmem_wait_ld();
  #pragma unroll
            for (int e = 0; e < 32; ++e) o_acc[c * 32 + e] = fmaf(o_acc[c * 32 + e], alpha_prev, __uint_as_float(v[e]));
          }
        }
        // pass 2: P = 2^(s * scale_log2 - m_new) as bf16 over the consumed S columns, row sum
        float sum8[8];
  #pragma unroll
        for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
  #pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(t_s + c * 32, v);
          tmem_wait_ld();
          float p[32];
          if (need_mask) {
  #pragma unroll
            for (int e = 0; e < 32; ++e)
              p[e] = (k0 + c * 32 + e < lim) ? ex2_approx(fmaf(__uint_as_float(v[e]), sl2, -msub)) : 0.f;
          } else {
  #pragma unroll
            for (int e = 0; e < 32; ++e) p[e] = ex2_approx(fmaf(__uint_as_float(v[e]), sl2, -msub));
          }
          uint32_t pk[16];
  #pragma unroll
          for (int e = 0; e < 16; ++e) {
            sum8[e & 7] += p[2 * e] + p[2 * e + 1];
            pk[e] = pack_bf16x2(p[2 * e], p[2 * e + 1]);
          }
          tmem_st16(t_s + c * 16, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        bar_arrive(p_full);
        const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
        l = l * alpha + sum;
        m = m_new;
        alpha_prev = alpha;
      }
      // the tile's last O' is folded in after its PV
      if (ok && x.nkv >= 1 && wait_bar(o_full, (jj - 1) & 1, err, 18)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(t_s + C_O + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o_acc[c * 32 + e] = fmaf(o_acc[c * 32 + e], alpha_prev, __uint_as_float(v[e]));
        }
      }
      if (ok && q < a.T) {
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        bf16* orow = a.o + (int64_t)(x.row0 + q) * a.ld_o + x.h * HD;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
          float tt[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tt[e] = o_acc[c * 8 + e] * inv;
          *reinterpret_cast<BF16x8*>(orow + c * 8) = float_to_bf16x8(tt);
        }
        // natural-log lse of the scaled scores: (m + log2 l) / log2(e)
        a.lse[((int64_t)x.b * a.H + x.h) * a.T + q] = (l > 0.f) ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
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

template <int HD>
cudaError_t launch_fwd(const CUtensorMap& tm, const AttnFwdArgs& args, int nqb, cudaStream_t st) {
  auto kern = flash_fwd_kernel<HD>;
  constexpr size_t smem = FwdSmem<HD>::TOTAL;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = args.B * args.H * nqb;
  launch_pdl(kern, std::min(tiles, 2 * persistent_sms()), kAttnThreads, smem, st, tm, args);
  return cudaGetLastError();
}

}  // namespace

int* attn_err_word() {
  static std::atomic<int*> slots[64];
  return device_symbol_address(slots, g_attn_err);
}

int attn_error_code(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_err, &z, sizeof(int));
  }
  return v;
}

// qkv: (B*T, ld_qkv) bf16 packed post-RoPE rows ((H + 2*KV) * hd columns used);
// o: (B*T, H*hd) bf16; lse: (B, H, T) fp32.
cudaError_t flash_attn_fwd(const void* qkv, int64_t ld_qkv, void* o, float* lse, int B, int T, int H, int KV, int hd,
                           bool causal, float scale, cudaStream_t st) {
  LLMT_REQUIRE(hd == 64 || hd == 128, "flash_attn_fwd: head dim must be 64 or 128");
  LLMT_REQUIRE(KV > 0 && H % KV == 0, "flash_attn_fwd: H must be a multiple of KV");
  LLMT_REQUIRE(tma_ok(qkv, ld_qkv, 2), "flash_attn_fwd: qkv pitch/alignment not TMA-legal");
  if (B == 0 || T == 0) return cudaSuccess;
  AttnFwdArgs args{};
  args.o = static_cast<bf16*>(o);
  args.lse = lse;
  args.B = B;
  args.T = T;
  args.H = H;
  args.KV = KV;
  args.ld_o = H * hd;
  args.scale_log2 = scale * 1.4426950408889634f;
  args.causal = causal ? 1 : 0;
  args.err = attn_err_word();
  alignas(64) CUtensorMap tm;
  LLMT_REQUIRE(make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)(H + 2 * KV) * hd,
                            (uint64_t)B * T, ld_qkv, 64, 128),
               "flash_attn_fwd: tensor map rejected");
  const int nqb = (int)cdiv(T, kBlockM);
  return hd == 64 ? launch_fwd<64>(tm, args, nqb, st) : launch_fwd<128>(tm, args, nqb, st);
}

}  // namespace llmt

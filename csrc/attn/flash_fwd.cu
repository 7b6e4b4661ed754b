// Causal flash attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's F.scaled_dot_product_attention(is_causal=True) (bench_train.py:141-142)
// and its output transpose copy (bench_train.py:149): q, k, v are read by TMA straight from the
// packed post-RoPE qkv rows (B*T, (H + 2*KV) * hd) and o is written as (B*T, H*hd), the layout
// the wo GEMM consumes. Online softmax (Milakov & Gimelshein 2018; FlashAttention, Dao et al.).
//
// One CTA per (batch*head, 128-query block); heaviest causal blocks are scheduled first.
//   warp 0     TMA producer: Q once, K/V blocks of 128 keys through a 2-stage ring
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S_j  = Q K_j^T        (M=128, N=128, K=hd)  -> TMEM S[j%2]
//                O'_j = P_j V_j        (M=128, N=hd,  K=128) -> TMEM O[j%2]
//              S_{j+1} is issued before O'_j so the tensor core works while softmax runs
//   warps 2-5  one thread per query row: two passes over S_j in TMEM (row max, then
//              exp2 and the row sum), P_j written as bf16 into 128B-swizzled shared memory
//              (the K-major A operand of the PV MMA), and O accumulated in registers:
//              O = O * exp2(m_old - m_new) + O'_j.
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
constexpr int kStages = 2;
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

// Byte offset of 16-byte unit `u` (0..15 over 128 bf16 columns) of row r in a K-major
// 128-row tile stored as two 64-column SW128 chunks of 16 KB.
__device__ __forceinline__ uint32_t sw128_row_unit(int r, int u) {
  return (uint32_t)((u >> 3) * 16384 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

template <int HD>
struct FwdSmem {
  static constexpr uint32_t Q_BYTES = kBlockM * HD * 2;
  static constexpr uint32_t KV_BYTES = kBlockN * HD * 2;
  static constexpr uint32_t P_BYTES = kBlockM * kBlockN * 2;
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = Q_OFF + Q_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + kStages * KV_BYTES;
  static constexpr uint32_t P_OFF = V_OFF + kStages * KV_BYTES;
  static constexpr uint32_t BAR_OFF = P_OFF + 2 * P_BYTES;
  static constexpr uint32_t TOTAL = BAR_OFF + 256 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnFwdArgs a) {
  using L = FwdSmem<HD>;
  constexpr int TMEM_COLS = 512;  // S[2] at 0/128, O[2] at 256/256+HD
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;       // [kStages]
  uint64_t* v_full = bars + 3;       // [kStages]
  uint64_t* kv_empty = bars + 5;     // [kStages]
  uint64_t* s_full = bars + 7;       // [2]
  uint64_t* s_empty = bars + 9;      // [2]
  uint64_t* p_full = bars + 11;      // [2]
  uint64_t* p_empty = bars + 13;     // [2]
  uint64_t* o_full = bars + 15;      // [2]
  uint64_t* o_empty = bars + 17;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int nqb = gridDim.y;
  const int qb = nqb - 1 - blockIdx.y;
  const int q0 = qb * kBlockM;
  const int kvh = h / (a.H / a.KV);
  const int nkv = a.causal ? min(qb + 1, (int)cdiv(a.T, kBlockN)) : (int)cdiv(a.T, kBlockN);
  const int row0 = b * a.T;  // first packed row of this sequence
  int* err = a.err;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&v_full[s], 1);
      bar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      bar_init(&s_full[i], 1);
      bar_init(&s_empty[i], 128);
      bar_init(&p_full[i], 128);
      bar_init(&p_empty[i], 1);
      bar_init(&o_full[i], 1);
      bar_init(&o_empty[i], 128);
    }
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
      const int qcol = h * HD, kcol = (a.H + kvh) * HD, vcol = (a.H + a.KV + kvh) * HD;
      bar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) tma_load_2d(smem + L::Q_OFF + c * 16384, &tm_qkv, q_full, qcol + c * 64, row0 + q0);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kStages;
        if (!wait_bar(&kv_empty[s], ((j / kStages) & 1) ^ 1, err, 11)) break;
        bar_arrive_expect_tx(&k_full[s], L::KV_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(smem + L::K_OFF + s * L::KV_BYTES + c * 16384, &tm_qkv, &k_full[s], kcol + c * 64, row0 + j * kBlockN);
        bar_arrive_expect_tx(&v_full[s], L::KV_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(smem + L::V_OFF + s * L::KV_BYTES + c * 16384, &tm_qkv, &v_full[s], vcol + c * 64, row0 + j * kBlockN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBlockM, HD, false, true);
      const uint32_t q_addr = smem_u32(smem + L::Q_OFF);
      bool ok = wait_bar(q_full, 0, err, 12);
      auto issue_pv = [&](int i) -> bool {
        const int s = i % kStages, pb = i & 1;
        if (!wait_bar(&v_full[s], (i / kStages) & 1, err, 13)) return false;
        if (!wait_bar(&p_full[pb], (i >> 1) & 1, err, 14)) return false;
        if (!wait_bar(&o_empty[pb], ((i >> 1) & 1) ^ 1, err, 15)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + L::P_OFF + pb * L::P_BYTES);
        const uint32_t v_addr = smem_u32(smem + L::V_OFF + s * L::KV_BYTES);
#pragma unroll
        for (int k = 0; k < kBlockN / 16; ++k) {
          const uint64_t ad = make_sw128_desc(p_addr + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(v_addr + k * 2048, 16384, 1024);
          mma_f16(tmem + 256 + pb * HD, ad, bd, idesc_o, k > 0 ? 1u : 0u);
        }
        mma_commit(&o_full[pb]);
        mma_commit(&p_empty[pb]);
        mma_commit(&kv_empty[s]);
        return true;
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % kStages, sb = j & 1;
        if (!wait_bar(&k_full[s], (j / kStages) & 1, err, 16)) { ok = false; break; }
        if (!wait_bar(&s_empty[sb], ((j >> 1) & 1) ^ 1, err, 17)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::K_OFF + s * L::KV_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_f16(tmem + sb * 128, make_sw128_desc(q_addr + off, 16, 1024), make_sw128_desc(k_addr + off, 16, 1024),
                  idesc_s, k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nkv >= 1) issue_pv(nkv - 1);
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the block
    const int q = q0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    float o_acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o_acc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    uint8_t* p_base = smem + L::P_OFF;
    bool ok = true;

    auto consume_o = [&](int i, float alpha) -> bool {
      const int pb = i & 1;
      if (!wait_bar(&o_full[pb], (i >> 1) & 1, err, 18)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + 256 + pb * HD + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o_acc[c * 32 + e] = o_acc[c * 32 + e] * alpha + __uint_as_float(v[e]);
      }
      tc_fence_before();
      bar_arrive(&o_empty[pb]);
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      if (!wait_bar(&s_full[sb], (j >> 1) & 1, err, 19)) { ok = false; break; }
      tc_fence_after();
      const int k0 = j * kBlockN;
      const bool need_mask = (a.causal && k0 + kBlockN - 1 > q0) || (k0 + kBlockN > a.T);
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + sb * 128 + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = k0 + c * 32 + e;
          const bool valid = !need_mask || (key < a.T && (!a.causal || key <= q));
          if (valid) mx = fmaxf(mx, __uint_as_float(v[e]));
        }
      }
      const float m_new = fmaxf(m, mx * a.scale_log2);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
      const float msub = (m_new == -INFINITY) ? 0.f : m_new;
      // pass 2: probabilities -> bf16 P tile (swizzled), row sum
      if (!wait_bar(&p_empty[sb], ((j >> 1) & 1) ^ 1, err, 20)) { ok = false; break; }
      uint8_t* prow = p_base + sb * L::P_BYTES;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + sb * 128 + c * 32, v);
        tmem_wait_ld();
        float p[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = k0 + c * 32 + e;
          const bool valid = !need_mask || (key < a.T && (!a.causal || key <= q));
          p[e] = valid ? exp2f(__uint_as_float(v[e]) * a.scale_log2 - msub) : 0.f;
          sum += p[e];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          BF16x8 pk = float_to_bf16x8(p + u * 8);
          *reinterpret_cast<BF16x8*>(prow + sw128_row_unit(r, c * 4 + u)) = pk;
        }
      }
      tc_fence_before();
      bar_arrive(&s_empty[sb]);
      fence_proxy_async_smem();
      bar_arrive(&p_full[sb]);
      l = l * alpha + sum;
      m = m_new;
      if (j >= 1 && !consume_o(j - 1, alpha_prev)) { ok = false; break; }
      alpha_prev = alpha;
    }
    if (ok && nkv >= 1) ok = consume_o(nkv - 1, alpha_prev);
    if (q < a.T) {
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      bf16* orow = a.o + (int64_t)(row0 + q) * a.ld_o + h * HD;
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        float t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = o_acc[c * 8 + e] * inv;
        *reinterpret_cast<BF16x8*>(orow + c * 8) = float_to_bf16x8(t);
      }
      // natural-log lse of the scaled scores: (m + log2 l) / log2(e)
      a.lse[((int64_t)b * a.H + h) * a.T + q] = (l > 0.f) ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
  }
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
  dim3 grid(args.B * args.H, nqb);
  kern<<<grid, kAttnThreads, smem, st>>>(tm, args);
  return cudaGetLastError();
}

}  // namespace

int* attn_err_word() {
  static int* p[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!p[dev]) cudaGetSymbolAddress(reinterpret_cast<void**>(&p[dev]), g_attn_err);
  return p[dev];
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

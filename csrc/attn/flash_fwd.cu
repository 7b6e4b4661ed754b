// Causal flash attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's F.scaled_dot_product_attention(is_causal=True) (bench_train.py:141-142)
// and its output transpose copy (bench_train.py:149): q, k, v are read by TMA straight from the
// packed post-RoPE qkv rows (B*T, (H + 2*KV) * hd) and o is written as (B*T, H*hd), the layout
// the wo GEMM consumes. Online softmax (Milakov & Gimelshein 2018; FlashAttention, Dao et al.).
//
// One persistent CTA per SM walks (batch*head, 256-query) tiles, heaviest causal tiles first, in
// a snake order. A tile is two 128-row query blocks, A and B, that share every K/V block; each
// has its own softmax warpgroup, so one block's softmax runs while the tensor core works on the
// other's ("ping-pong"):
//   warp 0     TMA producer: the tile's Q pair (double-buffered at head dim 64, so the next
//              tile's Q lands during this one) and 128-key K / V blocks through a ring
//   warp 1     TMEM allocator and MMA issuer (the warp runs the loop, one elected lane
//              issues), per key block j:
//                S_A = Q_A K_j^T, S_B = Q_B K_j^T      (SS form, M=128, N=128, K=hd)
//                O_A += P_A V_j,  O_B += P_B V_j       (TS form: P read from TMEM)
//              the next block's S is issued as soon as the softmax has read this block's S
//              out of TMEM, so score MMAs run ahead of the softmax
//   warps 2-5  softmax of block A, warps 6-9 of block B: one thread per query row holds the
//              row's 128 scores in registers; row max (three-input max), P = 2^(S*scale*log2e
//              - m) split between the SFU and an FMA-pipe polynomial, row sum, P packed to
//              bf16 in registers before the wait for the previous P.V, then stored to TMEM. O stays in TMEM: the running max is only moved (and O, l
//              rescaled in place) when it grows by more than 2^8, so most blocks skip the
//              rescale; O and l always refer to the same max, so the result is exact.
//              After a tile's last block the same warps normalise O and write o and lse.
// TMEM (512 columns): S_A, S_B 128 each; O_A, O_B hd each; at hd 64 P_A, P_B 64 each (bf16
// pairs), at hd 128 P is written over the block's own S columns (the next S then waits for the
// P.V that reads them).
// GQA: query head h reads key/value head h / (H / KV). Keys past T or past the query
// (causal) are masked. Saves lse (B, H, T) in natural-log units for the backward.
#include "../common/common.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.h"

namespace llmt {
int* attn_err_word();
namespace {

using namespace sm100;

constexpr int kBlockM = 128;   // query rows per softmax warpgroup
constexpr int kBlockN = 128;   // keys per K/V block
constexpr int kTileM = 256;    // query rows per tile (blocks A and B)
// TMA warp, MMA warp, two softmax warpgroups. Ten warps leave 168 registers a thread (three warps
// share a 16K-register SM sub-partition), enough for a row of 128 scores plus its P.
constexpr int kAttnThreads = 320;
constexpr float kRescaleLog2 = 8.f;  // move the running max only when it grows by more than 2^8
// One exponential pair in kPolyEvery runs as the FMA-pipe polynomial (ex2_poly), 0 = none. At head
// dim 64 the softmax is bound by the SFU (an event trace of one CTA: about 2,400 cycles per
// 128-key block with every exponential on the SFU); a quarter on the FMA pipe balances the SFU
// against the extra issue slots the polynomial costs.
constexpr int kPolyEvery = 4;

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
  static constexpr int QST = HD == 64 ? 2 : 1;   // Q pair buffers
  static constexpr int KVST = HD == 64 ? 3 : 2;  // K / V ring stages
  static constexpr uint32_t QB_BYTES = kBlockM * HD * 2;  // one 128-row Q block
  static constexpr uint32_t KV_BYTES = kBlockN * HD * 2;
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = Q_OFF + QST * 2 * QB_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + KVST * KV_BYTES;
  // O staging: one 32-row x 64-column bf16 box (4 KB, 128B swizzle) per softmax warp
  static constexpr uint32_t OST_OFF = V_OFF + KVST * KV_BYTES;
  static constexpr uint32_t BAR_OFF = OST_OFF + 8 * 4096;
  static constexpr uint32_t TOTAL = BAR_OFF + 256 + 1024;
  static_assert(TOTAL <= 232448, "attention forward shared memory exceeds the per-CTA limit");
};

__device__ __forceinline__ int fwd_snake(int r, int i, int G) { return r * G + ((r & 1) ? (G - 1 - i) : i); }

// Number of 128-key blocks block `half` (0 = A, 1 = B) of a tile starting at query q0 reads.
__device__ __forceinline__ int fwd_nkv(int q0, int half, int T, int causal) {
  const int qb0 = q0 + half * kBlockM;
  if (qb0 >= T) return 0;
  const int nall = (int)cdiv(T, kBlockN);
  return causal ? min(qb0 / kBlockN + 1, nall) : nall;
}

// VARIANT 0: the kernel. 1: the scaling FMA and the row sum as packed fp32 pairs (fewer
// instructions, more register pressure). 2: a timing skeleton with the softmax arithmetic
// replaced by constants (wrong results; it measures the MMA / TMA / barrier structure alone).
// 3: as 2, and the softmax warps do not touch TMEM either.
// Chosen at run time with LLMT_ATTN_VARIANT for measurements only.
template <int HD, int VARIANT>
__global__ void __launch_bounds__(kAttnThreads, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_o,
                 const AttnFwdArgs a) {
  pdl_wait();
  using L = FwdSmem<HD>;
  constexpr int QST = L::QST;
  constexpr int KVST = L::KVST;
  constexpr bool kSepP = HD == 64;  // P in its own TMEM columns (else over S)
  // TMEM columns of half w: S, O and P
  auto c_s = [](int w) -> uint32_t { return w ? 128u : 0u; };
  auto c_o = [](int w) -> uint32_t { return w ? 256u + HD : 256u; };
  auto c_p = [](int w) -> uint32_t { return kSepP ? (w ? 448u : 384u) : (w ? 128u : 0u); };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* k_full = bars + 0;        // [KVST]
  uint64_t* v_full = bars + 3;        // [KVST]
  uint64_t* kv_empty = bars + 6;      // [KVST]
  uint64_t* q_full = bars + 9;        // [QST]
  uint64_t* q_empty = bars + 11;      // [QST]
  uint64_t* s_full = bars + 13;       // [2] S of block A / B in TMEM
  uint64_t* s_free = bars + 15;       // [2] 128 arrivals: the softmax has read S (separate-P mode)
  uint64_t* p_full = bars + 17;       // [2] 128 arrivals: P written (and O rescaled)
  uint64_t* o_done = bars + 19;       // [2] the P.V of the last issued block has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_bh = a.B * a.H;
  const int npair = (int)cdiv(a.T, kTileM);
  const int n_tiles = n_bh * npair;
  const int G = gridDim.x;
  int* err = a.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < KVST; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&v_full[s], 1);
      bar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < QST; ++s) {
      bar_init(&q_full[s], 1);
      bar_init(&q_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      bar_init(&s_full[w], 1);
      bar_init(&s_free[w], 128);
      bar_init(&p_full[w], 128);
      bar_init(&o_done[w], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  struct Tile {
    int b, h, q0, kvh, n[2], row0;
  };
  auto tile_of = [&](int t) {
    Tile x;
    const int pr = npair - 1 - t / n_bh;  // most key blocks first
    const int bh = t % n_bh;
    x.b = bh / a.H;
    x.h = bh % a.H;
    x.q0 = pr * kTileM;
    x.kvh = x.h / (a.H / a.KV);
    x.n[0] = fwd_nkv(x.q0, 0, a.T, a.causal);
    x.n[1] = fwd_nkv(x.q0, 1, a.T, a.causal);
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
        bar_arrive_expect_tx(&q_full[qs], 2 * L::QB_BYTES);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + L::Q_OFF + (qs * 2 + hb) * L::QB_BYTES + c * 16384, &tm_qkv, &q_full[qs],
                        qcol + c * 64, x.row0 + x.q0 + hb * kBlockM);
        const int nmax = max(x.n[0], x.n[1]);
        for (int j = 0; j < nmax; ++j, ++jj) {
          const int s = jj % KVST;
          if (!wait_bar(&kv_empty[s], ((jj / KVST) & 1) ^ 1, err, 11)) { ok = false; break; }
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
    {  // the whole warp runs the issue loop; one elected lane issues each MMA
      constexpr uint32_t idesc_s = make_idesc_bf16(kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBlockM, HD, false, true);
      // TMEM base and shared-memory descriptors as warp-uniform values (kept in uniform registers,
      // which the MMA instructions read directly); per-MMA descriptors are the base plus an offset
      const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);
      int jj = 0, tl = 0;
      int cnt[2] = {0, 0};  // blocks issued per half, over all tiles (barrier phases)
      bool ok = true;
      // S_w = Q_w K^T into S columns of half w; waits until the half's previous S was read
      // (separate P) or its previous P.V completed (P over S).
      // g: the half's global block index of this S
      auto issue_s = [&](int w, int g, uint32_t q_addr, uint32_t k_addr) -> bool {
        if (g > 0) {
          if (kSepP) {
            if (!wait_bar_w(&s_free[w], (g - 1) & 1, err, 15)) return false;
          } else {
            if (!wait_bar_w(&o_done[w], (g - 1) & 1, err, 15)) return false;
          }
        }
        tc_fence_after();
        const uint64_t qd = make_sw128_desc(q_addr, 16, 1024), kd = make_sw128_desc(k_addr, 16, 1024);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
          umma_f16(tm + c_s(w), qd + off, kd + off, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
        return true;
      };
      for (int r = 0; ok; ++r, ++tl) {
        const int t = fwd_snake(r, blockIdx.x, G);
        if (t >= n_tiles) break;
        const Tile x = tile_of(t);
        const int qs = tl % QST;
        if (!wait_bar_w(&q_full[qs], (tl / QST) & 1, err, 12)) break;
        const uint32_t q_addr0 = smem_u32(smem + L::Q_OFF + (qs * 2) * L::QB_BYTES);
        const uint32_t q_addr1 = q_addr0 + L::QB_BYTES;
        const int nmax = max(x.n[0], x.n[1]);
        // S of key block 0
        {
          const int s0 = jj % KVST;
          if (!wait_bar_w(&k_full[s0], (jj / KVST) & 1, err, 16)) break;
          const uint32_t k_addr = smem_u32(smem + L::K_OFF + s0 * L::KV_BYTES);
          if (x.n[0] > 0) ok = issue_s(0, cnt[0], q_addr0, k_addr);
          if (ok && x.n[1] > 0) ok = issue_s(1, cnt[1], q_addr1, k_addr);
          if (!ok) break;
          if (nmax == 1) umma_commit(&q_empty[qs]);
        }
        for (int j = 0; j < nmax && ok; ++j, ++jj) {
          const int s = jj % KVST;
          if (kSepP && j + 1 < nmax) {  // run the next block's scores ahead of this block's P.V
            const int s1 = (jj + 1) % KVST;
            if (!wait_bar_w(&k_full[s1], ((jj + 1) / KVST) & 1, err, 16)) { ok = false; break; }
            const uint32_t k_addr = smem_u32(smem + L::K_OFF + s1 * L::KV_BYTES);
            if (j + 1 < x.n[0]) ok = issue_s(0, cnt[0] + 1, q_addr0, k_addr);
            if (ok && j + 1 < x.n[1]) ok = issue_s(1, cnt[1] + 1, q_addr1, k_addr);
            if (!ok) break;
            if (j + 2 == nmax) umma_commit(&q_empty[qs]);  // the tile's last S has read its Q
          }
          if (!wait_bar_w(&v_full[s], (jj / KVST) & 1, err, 13)) { ok = false; break; }
          const uint32_t v_addr = smem_u32(smem + L::V_OFF + s * L::KV_BYTES);
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            if (j >= (w ? x.n[1] : x.n[0])) continue;
            if (!wait_bar_w(&p_full[w], cnt[w] & 1, err, 14)) { ok = false; break; }
            tc_fence_after();
            const uint64_t vd = make_sw128_desc(v_addr, 16384, 1024);
#pragma unroll
            for (int k = 0; k < kBlockN / 16; ++k)
              umma_f16_ts(tm + c_o(w), tm + c_p(w) + k * 8, vd + (uint64_t)(k * 2048 >> 4), idesc_o,
                          (j > 0 || k > 0) ? 1u : 0u);
            umma_commit(&o_done[w]);
            ++cnt[w];
          }
          if (!ok) break;
          umma_commit(&kv_empty[s]);
          if (!kSepP && j + 1 < nmax) {  // P over S: the next S waits for this block's P.V
            const int s1 = (jj + 1) % KVST;
            if (!wait_bar_w(&k_full[s1], ((jj + 1) / KVST) & 1, err, 16)) { ok = false; break; }
            const uint32_t k_addr = smem_u32(smem + L::K_OFF + s1 * L::KV_BYTES);
            if (j + 1 < x.n[0]) ok = issue_s(0, cnt[0], q_addr0, k_addr);
            if (ok && j + 1 < x.n[1]) ok = issue_s(1, cnt[1], q_addr1, k_addr);
            if (!ok) break;
            if (j + 2 == nmax) umma_commit(&q_empty[qs]);
          }
        }
      }
    }
  } else {
    // softmax warpgroups: warps 2-5 -> half A, 6-9 -> half B; TMEM lane quadrant = warp % 4
    const int w = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the block
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_off + c_s(w);
    const uint32_t t_o = tmem + lane_off + c_o(w);
    const uint32_t t_p = tmem + lane_off + c_p(w);
    const float sl2 = a.scale_log2;
    int cnt = 0;  // blocks of this half processed, over all tiles
    bool ok = true;
    for (int rr = 0; ok; ++rr) {
      const int t = fwd_snake(rr, blockIdx.x, G);
      if (t >= n_tiles) break;
      const Tile x = tile_of(t);
      const int nkv = w ? x.n[1] : x.n[0];
      if (nkv == 0) continue;
      const int qb0 = x.q0 + w * kBlockM;
      const int q = qb0 + r;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv; ++j, ++cnt) {
        if (!wait_bar(&s_full[w], cnt & 1, err, 19)) { ok = false; break; }
        tc_fence_after();
        uint32_t su[kBlockN];  // the row's scores (fp32 bits)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (VARIANT == 3) {
#pragma unroll
            for (int e = 0; e < 32; ++e) su[c * 32 + e] = __float_as_uint((float)(e + c));
          } else {
            tmem_ld32(t_s + c * 32, *reinterpret_cast<uint32_t(*)[32]>(su + c * 32));
          }
        }
        tmem_wait_ld();
        if (kSepP) {
          tc_fence_before();
          bar_arrive(&s_free[w]);  // the next block's S may be computed now
        }
        const int k0 = j * kBlockN;
        // keys allowed for this row: key < lim (causal: key <= q; always key < T)
        const int lim = a.causal ? min(q + 1, a.T) : a.T;
        const bool need_mask = k0 + kBlockN > (a.causal ? qb0 + 1 : a.T) || k0 + kBlockN > a.T;
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < kBlockN; ++e)
            if (k0 + e >= lim) su[e] = 0xff800000u;  // -inf
        }
        // row max: three-input max over key pairs, four independent chains
        auto sf = [&](int e) { return __uint_as_float(su[e]); };
        float mx4[4] = {sf(0), sf(1), sf(2), sf(3)};
#pragma unroll
        for (int e = 4; e < kBlockN; e += 8) {
          mx4[0] = max3f(mx4[0], sf(e), sf(e + 1));
          mx4[1] = max3f(mx4[1], sf(e + 2), sf(e + 3));
          mx4[2] = max3f(mx4[2], sf(e + 4), sf(e + 5));
          mx4[3] = max3f(mx4[3], sf(e + 6), sf(e + 7));
        }
        const float mx = VARIANT >= 2 ? 0.f : fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
        // move the running max (and rescale O and l) only if it grew by more than 2^8 in some row
        const bool grow = mx > m_used + kRescaleLog2;
        const bool rescale = __any_sync(0xffffffffu, grow);
        float alpha = 1.f;
        if (rescale) {
          const float m_new = fmaxf(m_used, mx);
          alpha = ex2_approx(m_used - m_new);  // m_used = -inf on the first block -> 0
          m_used = m_new;
        }
        const float msub = (m_used == -INFINITY) ? 0.f : m_used;
        // P = 2^(s * scale_log2 - m): one exponential pair in kPolyEvery on the FMA pipe, the rest
        // on the SFU; packed to bf16 pairs in registers
        const float2 sl2x2 = make_float2(sl2, sl2), negm = make_float2(-msub, -msub);
        float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        uint32_t pk[kBlockN / 2];
#pragma unroll
        for (int e = 0; e < kBlockN; e += 2) {
          const float2 xx = VARIANT == 1 ? fma2(make_float2(sf(e), sf(e + 1)), sl2x2, negm)
                                         : make_float2(fmaf(sf(e), sl2, -msub), fmaf(sf(e + 1), sl2, -msub));
          float2 pp;
          if (VARIANT >= 2) {
            pp = xx;
          } else if (kPolyEvery > 0 && (e >> 1) % kPolyEvery == kPolyEvery - 1) {
            pp.x = ex2_poly(xx.x);
            pp.y = ex2_poly(xx.y);
            if (need_mask) {  // the polynomial does not map -inf to 0
              pp.x = su[e] == 0xff800000u ? 0.f : pp.x;
              pp.y = su[e + 1] == 0xff800000u ? 0.f : pp.y;
            }
          } else {
            pp.x = ex2_approx(xx.x);
            pp.y = ex2_approx(xx.y);
          }
          if (VARIANT == 1) {
            sum2[(e >> 1) & 3] = add2(sum2[(e >> 1) & 3], pp);
          } else {
            sum2[(e >> 1) & 3].x += pp.x;
            sum2[(e >> 1) & 3].y += pp.y;
          }
          pk[e >> 1] = pack_bf16x2(pp.x, pp.y);
        }
        // P must exist before the wait below: the compiler would otherwise sink this arithmetic past
        // the wait, and the softmax would idle for the previous P.V before doing its work
#pragma unroll
        for (int i = 0; i < kBlockN / 2; ++i) asm volatile("" ::"r"(pk[i]));
        // The previous block's P.V has completed before O is rescaled or P rewritten: with P over S
        // this block's S was issued after it; with separate P it is waited for here.
        if (kSepP && j > 0 && !wait_bar(&o_done[w], (cnt - 1) & 1, err, 18)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (VARIANT != 3) tmem_st16(t_p + c * 16, *reinterpret_cast<uint32_t(*)[16]>(pk + c * 16));
        if (rescale && j > 0) {
#pragma unroll
          for (int c = 0; c < HD / 16; ++c) {
            uint32_t v[16];
            tmem_ld16(t_o + c * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st16(t_o + c * 16, v);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        bar_arrive(&p_full[w]);
        const float2 s01 = add2(sum2[0], sum2[1]), s23 = add2(sum2[2], sum2[3]);
        l = l * alpha + ((s01.x + s01.y) + (s23.x + s23.y));
      }
      if (!ok) break;
      // epilogue: the last P.V of the tile, then o = O / l and lse
      if (!wait_bar(&o_done[w], (cnt - 1) & 1, err, 20)) { ok = false; break; }
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      // A warp's 32 full rows leave through TMA stores of 32 x 64 bf16 boxes staged (128B swizzle)
      // in its own 4 KB slot: per-thread stores of 16-byte row pieces, 32 rows per instruction,
      // are many times slower. Rows of a ragged last block keep per-thread stores (rows past T
      // belong to the next sequence).
      const bool box = qb0 + quad * 32 + 32 <= a.T;  // warp-uniform
      uint8_t* stg = smem + L::OST_OFF + (warp - 2) * 4096;
      bf16* orow = a.o + (int64_t)(x.row0 + min(q, a.T - 1)) * a.ld_o + x.h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(t_o + c * 32, v);
        tmem_wait_ld();
        if (box) {
          if ((c & 1) == 0) {  // the slot's previous box must have been read by its TMA store
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float tt[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) tt[e] = __uint_as_float(v[u * 8 + e]) * inv;
            const int unit = (c & 1) * 4 + u;
            *reinterpret_cast<BF16x8*>(stg + lane * 128 + ((unit ^ (lane & 7)) << 4)) = float_to_bf16x8(tt);
          }
          if (c & 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tm_o, stg, x.h * HD + (c >> 1) * 64, x.row0 + qb0 + quad * 32);
              bulk_commit();
            }
          }
        } else if (q < a.T) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float tt[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) tt[e] = __uint_as_float(v[u * 8 + e]) * inv;
            *reinterpret_cast<BF16x8*>(orow + c * 32 + u * 8) = float_to_bf16x8(tt);
          }
        }
      }
      tc_fence_before();  // O may be overwritten by the next tile's first P.V after p_full
      // natural-log lse of the scaled scores: (m + log2 l) / log2(e)
      if (q < a.T)
        a.lse[((int64_t)x.b * a.H + x.h) * a.T + q] = (l > 0.f) ? (m_used + log2f(l)) * 0.69314718055994530942f
                                                               : -INFINITY;
    }
  }
  if (warp >= 2) {  // the softmax warps' O stores are complete before the CTA exits
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
  pdl_trigger();  // this CTA is done: the next kernel in the stream may be scheduled
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

template <int HD, int VARIANT>
cudaError_t launch_fwd_v(const CUtensorMap& tm, const CUtensorMap& tmo, const AttnFwdArgs& args, cudaStream_t st) {
  auto kern = flash_fwd_kernel<HD, VARIANT>;
  constexpr size_t smem = FwdSmem<HD>::TOTAL;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = args.B * args.H * (int)cdiv(args.T, kTileM);
  launch_pdl(kern, std::min(tiles, persistent_sms()), kAttnThreads, smem, st, tm, tmo, args);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_fwd(const CUtensorMap& tm, const CUtensorMap& tmo, const AttnFwdArgs& args, cudaStream_t st) {
  static const int variant = [] {
    const char* e = getenv("LLMT_ATTN_VARIANT");
    return e ? atoi(e) : 0;
  }();
  if (variant == 1) return launch_fwd_v<HD, 1>(tm, tmo, args, st);
  if (variant == 2) return launch_fwd_v<HD, 2>(tm, tmo, args, st);
  if (variant == 3) return launch_fwd_v<HD, 3>(tm, tmo, args, st);
  return launch_fwd_v<HD, 0>(tm, tmo, args, st);
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
  alignas(64) CUtensorMap tmo;  // 32-row x 64-column boxes of o for the TMA-store epilogue
  LLMT_REQUIRE(tma_ok(o, (int64_t)H * hd, 2) && make_tmap_2d(&tmo, o, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                                             (uint64_t)H * hd, (uint64_t)B * T, (uint64_t)H * hd, 64, 32),
               "flash_attn_fwd: output tensor map rejected");
  return hd == 64 ? launch_fwd<64>(tm, tmo, args, st) : launch_fwd<128>(tm, tmo, args, st);
}

}  // namespace llmt

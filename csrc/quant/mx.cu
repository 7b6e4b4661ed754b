// Block-scaled quantization for the MXFP8 and NVFP4 linears.
//
// Both formats scale small blocks along the GEMM's contraction dimension, so a linear needs its
// operands quantized along K for the forward (x, w), along N for the dgrad (dy, w^T) and along M
// for the wgrad (dy^T, x^T). One kernel reads a 64 x 64 tile of x once and writes, as asked, the
// row-wise copy q (blocks along cols) and the transposed copy qt (blocks along rows, through
// shared memory), each with its scales in the chunked layout the block-scaled GEMM loads:
// chunk = 128 rows x 4 scales, 512 bytes, row r at (r % 32) * 16 + ((r / 32) % 4) * 4, scale k
// at + k; chunks ordered [row tile][position along K].
//
// MXFP8 (OCP microscaling): e4m3 data, one ue8m0 scale 2^e per 32 values, e the smallest power
// with amax <= 448 * 2^e (so nothing saturates), found from amax's exponent and mantissa bits.
// NVFP4 follows the reference's recipe (kernels/lowp.py:110-138, :192-235): per-tensor decode
// scale g = amax / (6 * 448); per 16 values an e4m3 scale s = e4m3(min(bamax / (6 g), 448));
// v = x * (1 / (s g)) clamped to +-6 and rounded to e2m1 (0, 0.5, 1, 1.5, 2, 3, 4, 6): to nearest
// with ties down, or stochastically (dy) with 16-bit uniforms from Philox-4x32-10 (Salmon et al.,
// SC 2011); two values per byte, the first in the low nibble.
#include <cuda_fp8.h>

#include "../common/common.cuh"

namespace llmt {
namespace {

constexpr int kAmaxBlocks = 296;
constexpr int kThreads = 256;
constexpr int kTile = 64;

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* v);
template <>
__device__ __forceinline__ void load16<bf16>(const bf16* p, float* v) {
  bf16x8_to_float(*reinterpret_cast<const BF16x8*>(p), v);
  bf16x8_to_float(*reinterpret_cast<const BF16x8*>(p + 8), v + 8);
}
template <>
__device__ __forceinline__ void load16<float>(const float* p, float* v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = ld_f4(p + 4 * i);
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

__device__ __forceinline__ int64_t sf_off(int r, int c, int chunks) {
  return ((int64_t)(r >> 7) * chunks + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// ---------------------------------------------------------------- MXFP8
__device__ __forceinline__ int mx_exp(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int E = (int)((b >> 23) & 0xFF) - 127;
  if (!(amax > 0.f) || E == -127) return -127;  // zero or subnormal block: the smallest scale
  const int e = (b & 0x7FFFFFu) > 0x600000u ? E - 7 : E - 8;  // 448 = 1.75 * 2^8
  return e < -127 ? -127 : e;
}

// 16 values -> 16 e4m3 bytes scaled by 2^-e
__device__ __forceinline__ uint4 e4m3x16(const float* v, int e) {
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t lo =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * inv, v[4 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * inv, v[4 * i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
    w[i] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---------------------------------------------------------------- NVFP4
__device__ __forceinline__ uint4 philox(uint4 c, uint2 k) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

__device__ __forceinline__ float e2m1_mag(int i) {
  return i < 4 ? 0.5f * (float)i : (i == 4 ? 2.f : (i == 5 ? 3.f : (i == 6 ? 4.f : 6.f)));
}

// one 16-value block -> 8 bytes of e2m1 pairs and its e4m3 scale byte
__device__ __forceinline__ uint2 nvfp4_block(const float* v, float g, bool stochastic, uint64_t seed, int64_t idx0,
                                             uint8_t* scale_byte) {
  float bamax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bamax = fmaxf(bamax, fabsf(v[i]));
  const float s = fminf(__fdiv_rn(bamax, __fmul_rn(6.f, g)), 448.f);
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3);
  *scale_byte = (uint8_t)s8;
  __nv_fp8_e4m3 sv;
  sv.__x = s8;
  const float denom = __fmul_rn(static_cast<float>(sv), g);
  // the reference's quantizer multiplies by one reciprocal per block (lowp.py:213-214)
  const float inv = denom > 0.f ? __frcp_rn(denom) : 0.f;
  float u[16];
  if (stochastic) {
    // two 16-bit uniforms per 32-bit Philox output: 8 per call, 2 calls per block
    const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint64_t n = (uint64_t)idx0 + 8 * q;
      const uint4 r = philox(make_uint4((uint32_t)n, (uint32_t)(n >> 32), 0u, 0u), key);
      const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        u[8 * q + 2 * j] = (float)(w4[j] >> 16) * 1.52587890625e-5f;
        u[8 * q + 2 * j + 1] = (float)(w4[j] & 0xFFFFu) * 1.52587890625e-5f;
      }
    }
  }
  uint32_t code[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x = fminf(fmaxf(v[i] * inv, -6.f), 6.f);
    const float mag = fabsf(x);
    int id;
    if (stochastic) {
      const int lo = (mag >= 0.5f) + (mag >= 1.f) + (mag >= 1.5f) + (mag >= 2.f) + (mag >= 3.f) + (mag >= 4.f) +
                     (mag >= 6.f);
      const int hi = lo < 7 ? lo + 1 : 7;
      // grid steps are 0.5 below 2, 1 up to 4, then 2: the fraction is an exact power-of-two product
      const float frac = lo < 7 ? (mag - e2m1_mag(lo)) * (lo < 4 ? 2.f : (lo < 6 ? 1.f : 0.5f)) : 0.f;
      id = u[i] < frac ? hi : lo;
    } else {
      // nearest, ties down: count the midpoints strictly below mag
      id = (mag > 0.25f) + (mag > 0.75f) + (mag > 1.25f) + (mag > 1.75f) + (mag > 2.5f) + (mag > 3.5f) + (mag > 5.f);
    }
    code[i] = (uint32_t)id | ((x < 0.f && id > 0) ? 8u : 0u);
  }
  uint2 out = make_uint2(0u, 0u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out.x |= (code[2 * i] | (code[2 * i + 1] << 4)) << (8 * i);
    out.y |= (code[8 + 2 * i] | (code[8 + 2 * i + 1] << 4)) << (8 * i);
  }
  return out;
}

__device__ __forceinline__ float block_max(float m, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = m;
  __syncthreads();
  m = l < kThreads / 32 ? red[l] : 0.f;
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return __shfl_sync(0xffffffffu, m, 0);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) amax_partial_kernel(const T* __restrict__ x, int rows, int cols, int64_t ld,
                                                                float* __restrict__ partial) {
  pdl_wait();
  __shared__ float red[kThreads / 32];
  const int gpr = cols / 16;  // 16-element groups per row
  const int64_t n = (int64_t)rows * gpr;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  float m = 0.f;
  if (ld == cols) {  // contiguous: no row / column split (a 64-bit division per group costs more than the load)
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
      float v[16];
      load16(x + i * 16, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
    }
  } else {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {  // a row per CTA, its groups over the threads
      for (int i = threadIdx.x; i < gpr; i += kThreads) {
        float v[16];
        load16(x + (int64_t)r * ld + i * 16, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
      }
    }
  }
  m = block_max(m, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = m;
  pdl_trigger();
}

struct MxArgs {
  int rows, cols;
  int64_t ld;
  uint8_t* q;    // (rows, cols) MXFP8 / (rows, cols / 2) NVFP4, or null
  uint8_t* sf;
  int chunks;    // per 128-row tile of q
  uint8_t* qt;   // (cols, rows) / (cols, rows / 2), or null
  uint8_t* sft;
  int chunks_t;
  int interleave64;  // q rows: 64 of the first half, 64 of the second, ... (merged SwiGLU weight)
  const float* partial;  // NVFP4: amax partials of x
  float* g_out;
  int stochastic;
  uint64_t seed;
  const int64_t* seed_dev;  // optional: added to seed (a step counter kept on the device, so a
                            // captured CUDA graph draws new noise on every replay)
};

__device__ __forceinline__ int dest_row(int r, int rows, int il) {
  if (!il) return r;
  const int F = rows / 2;
  const int h = r >= F, o = r - h * F;
  return (o / 64) * 128 + h * 64 + (o % 64);
}

template <typename T, int KIND>
__global__ void __launch_bounds__(kThreads) mx_quant_kernel(const T* __restrict__ x, const MxArgs a) {
  pdl_wait();
  __shared__ float tile[kTile][kTile + 1];
  __shared__ float red[kThreads / 32];
  float g = 0.f;
  if constexpr (KIND == 3) {
    float m = 0.f;
    for (int i = threadIdx.x; i < kAmaxBlocks; i += kThreads) m = fmaxf(m, a.partial[i]);
    // amax / (6 * 448), evaluated as PyTorch does for a tensor over a Python scalar on CUDA:
    // times the float reciprocal of the scalar
    g = fmaxf(__fmul_rn(block_max(m, red), 1.f / 2688.f), 1e-30f);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *a.g_out = g;
  }
  const uint64_t seed = a.seed + (a.seed_dev ? (uint64_t)(*a.seed_dev) * 0x9E3779B97F4A7C15ull : 0ull);
  const int r0 = blockIdx.y * kTile, c0 = blockIdx.x * kTile;
  const int tr = threadIdx.x >> 2, tq = threadIdx.x & 3;
  const int r = r0 + tr, c = c0 + tq * 16;
  float v[16];
  const bool valid = r < a.rows && c < a.cols;
  if (valid) {
    load16(x + (int64_t)r * a.ld + c, v);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
  }
  if (a.q) {
    const int dr = dest_row(r, a.rows, a.interleave64);
    if constexpr (KIND == 2) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));  // the pair holding one 32-value block
      const int e = mx_exp(m);
      if (valid) {
        *reinterpret_cast<uint4*>(a.q + (int64_t)dr * a.cols + c) = e4m3x16(v, e);
        if ((tq & 1) == 0) a.sf[sf_off(dr, c >> 5, a.chunks)] = (uint8_t)(e + 127);
      }
    } else {
      uint8_t sb;
      const uint2 p = nvfp4_block(v, g, a.stochastic, seed, (int64_t)r * a.cols + c, &sb);
      if (valid) {
        *reinterpret_cast<uint2*>(a.q + (int64_t)dr * (a.cols / 2) + c / 2) = p;
        a.sf[sf_off(dr, c >> 4, a.chunks)] = sb;
      }
    }
  }
  if (a.qt) {
#pragma unroll
    for (int i = 0; i < 16; ++i) tile[tr][tq * 16 + i] = v[i];
    __syncthreads();
    const int cc = threadIdx.x >> 2, rq = threadIdx.x & 3;  // column of x, quarter of the tile's rows
    float w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = tile[rq * 16 + i][cc];
    const int qr = c0 + cc, qc = r0 + rq * 16;  // row / first column of qt
    const bool tvalid = qr < a.cols && qc < a.rows;
    if constexpr (KIND == 2) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(w[i]));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      const int e = mx_exp(m);
      if (tvalid) {
        *reinterpret_cast<uint4*>(a.qt + (int64_t)qr * a.rows + qc) = e4m3x16(w, e);
        if ((rq & 1) == 0) a.sft[sf_off(qr, qc >> 5, a.chunks_t)] = (uint8_t)(e + 127);
      }
    } else {
      uint8_t sb;
      const uint2 p = nvfp4_block(w, g, a.stochastic, seed ^ 0x5bd1e995u, (int64_t)qr * a.rows + qc, &sb);
      if (tvalid) {
        *reinterpret_cast<uint2*>(a.qt + (int64_t)qr * (a.rows / 2) + qc / 2) = p;
        a.sft[sf_off(qr, qc >> 4, a.chunks_t)] = sb;
      }
    }
  }
  pdl_trigger();
}

// chunks per 128-row tile for a row of `cols` elements: k-blocks of 128 bytes x chunks per k-block
int chunks_for(int kind, int cols) {
  return kind == 2 ? (int)cdiv(cols, 128) : 4 * (int)cdiv(cols, 256);
}

template <typename T>
void launch_mx(int kind, const T* x, MxArgs& a, float* scratch, cudaStream_t st) {
  dim3 grid((unsigned)cdiv(a.cols, kTile), (unsigned)cdiv(a.rows, kTile));
  if (kind == 3) {
    launch_pdl(amax_partial_kernel<T>, kAmaxBlocks, kThreads, 0, st, x, a.rows, a.cols, a.ld, scratch);
    a.partial = scratch;
    launch_pdl(mx_quant_kernel<T, 3>, grid, kThreads, 0, st, x, a);
  } else {
    launch_pdl(mx_quant_kernel<T, 2>, grid, kThreads, 0, st, x, a);
  }
}

}  // namespace

int64_t mx_sf_bytes(int kind, int rows, int cols) { return cdiv(rows, 128) * (int64_t)chunks_for(kind, cols) * 512; }

cudaError_t mx_quant(int kind, const void* x, bool x_f32, int rows, int cols, int64_t ld, void* q, void* sf, void* qt,
                     void* sft, float* g_out, float* scratch, bool interleave64, bool stochastic, uint64_t seed,
                     const int64_t* seed_dev, cudaStream_t st) {
  LLMT_REQUIRE(kind == 2 || kind == 3, "mx_quant: kind must be 2 (MXFP8) or 3 (NVFP4)");
  if (kind == 2)
    LLMT_REQUIRE(cols % 32 == 0 && (!qt || rows % 32 == 0), "mx_quant: MXFP8 needs dims that are multiples of 32");
  else
    LLMT_REQUIRE(cols % 64 == 0 && rows % 64 == 0 && g_out && scratch,
                 "mx_quant: NVFP4 needs dims that are multiples of 64 and a decode-scale output");
  LLMT_REQUIRE(ld % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0, "mx_quant: x needs 16-byte alignment");
  LLMT_REQUIRE((!q || sf) && (!qt || sft), "mx_quant: every output needs its scale buffer");
  LLMT_REQUIRE(!interleave64 || (rows % 128 == 0), "mx_quant: interleaving needs rows a multiple of 128");
  if (rows == 0 || cols == 0) return cudaSuccess;
  MxArgs a{};
  a.rows = rows;
  a.cols = cols;
  a.ld = ld;
  a.q = static_cast<uint8_t*>(q);
  a.sf = static_cast<uint8_t*>(sf);
  a.chunks = chunks_for(kind, cols);
  a.qt = static_cast<uint8_t*>(qt);
  a.sft = static_cast<uint8_t*>(sft);
  a.chunks_t = chunks_for(kind, rows);
  a.interleave64 = interleave64 ? 1 : 0;
  a.g_out = g_out;
  a.stochastic = stochastic ? 1 : 0;
  a.seed = seed;
  a.seed_dev = seed_dev;
  if (x_f32) launch_mx(kind, static_cast<const float*>(x), a, scratch, st);
  else launch_mx(kind, static_cast<const bf16*>(x), a, scratch, st);
  return cudaGetLastError();
}

}  // namespace llmt

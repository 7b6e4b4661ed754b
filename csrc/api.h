// Plain C++ launch API of the llmt sm_100a kernels (no torch types).
//
// Every .cu translation unit implements its launchers against raw device pointers and a
// cudaStream_t; the PyTorch glue (bindings.cpp) validates tensors and calls these. Keeping
// torch headers out of the CUDA units keeps device compiles to seconds, and gives callers
// outside PyTorch the same entry points. Launchers return cudaSuccess or an error; for
// argument errors they return cudaErrorInvalidValue and leave a message in last_error().
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmt {

const char* last_error();
void set_last_error(const char* msg);
int sm_count();
// SMs reserved for kernels running beside the persistent ones; persistent grids use the rest.
void set_reserved_sms(int n);
int reserved_sms();
int persistent_sms();
// Bounds-checked build: each translation unit registers the reader of its out-of-range record;
// bounds_error() returns the first non-zero record (bit 63 | site << 40 | index) or 0, and
// bounds_checking() says whether this module was built with the checks.
int register_bounds_reader(unsigned long long (*reader)(bool reset));
unsigned long long bounds_error(bool reset);
bool bounds_checking();
#ifdef LLMT_DEBUG_BOUNDS
cudaError_t bounds_probe(float* buf, int64_t n, int64_t i, cudaStream_t st);  // common/bounds_probe.cu
#endif

// ---------------------------------------------------------------- RMSNorm
cudaError_t add_rmsnorm_fwd(const void* a_bf16, const float* r, const float* w, void* y_bf16, float* s, float* rstd,
                            int64_t N, int D, float eps, cudaStream_t st);
int rmsnorm_bwd_partials(int64_t N, int D);  // rows of the dw partial buffer the backward needs
cudaError_t rmsnorm_bwd(const void* dy_bf16, const float* s, const float* w, const float* rstd, const float* ds_in,
                        float* ds, void* ds16, float* dw_part, float* dw, unsigned* ticket, int64_t N, int D,
                        int accumulate, cudaStream_t st);

// ---------------------------------------------------------------- elementwise
cudaError_t swiglu_fwd(const void* g, const void* u, int64_t ldgu, void* h, int64_t ldh, int64_t rows, int F,
                       cudaStream_t st);
cudaError_t swiglu_bwd(const void* dh, int64_t lddh, const void* g, const void* u, int64_t ldgu, void* dg, void* du,
                       int64_t lddgu, int64_t rows, int F, cudaStream_t st);
cudaError_t rope_inplace(void* qkv, const float* cos_t, const float* sin_t, int64_t N, int T, int n_rot_heads, int hd,
                         int64_t ld, bool backward, cudaStream_t st);
// W holds vocabulary rows [v0, v0 + V); `partial` (a vocabulary-parallel shard) gives zero rows
// for ids outside it instead of flagging them.
cudaError_t embedding_fwd(const int64_t* idx, const float* W, float* x, int64_t N, int d, int64_t V, int64_t v0,
                          bool partial, int* err, cudaStream_t st);
cudaError_t embedding_bwd(const int64_t* idx, const float* dx, float* dW, int64_t N, int d, int64_t V, int64_t v0,
                          cudaStream_t st);

// ---------------------------------------------------------------- optimizer
struct AdamHyper {
  float b1, b2, eps, wd, grad_scale;
};
cudaError_t adamw_step(float* p, float* g, float* m, float* v, void* p16, int64_t n, const float* lr,
                       const int* step, AdamHyper h, bool zero_grad, cudaStream_t st, int max_blocks = 0);
cudaError_t cast_bf16(const float* x, void* y, int64_t n, cudaStream_t st, int max_blocks = 0);

// ---------------------------------------------------------------- cross entropy rows
cudaError_t ce_fwd_rows(const void* logits, int64_t ld, const int64_t* tgt, float* lse, float* loss, int64_t R, int V,
                        cudaStream_t st);
cudaError_t ce_bwd_rows(void* logits, int64_t ld, const int64_t* tgt, const float* lse, const float* grad_out,
                        float scale, int64_t R, int V, cudaStream_t st);
cudaError_t ce_combine(const float* part, const float* tlogit, const int64_t* tgt, float* lse, float* loss, int M,
                       int nblk, int V, cudaStream_t st);

// ---------------------------------------------------------------- GEMM
enum EpiKind : int {
  EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_SWIGLU_BWD = 3, EPI_ROPE = 4, EPI_CE_FWD = 5, EPI_CE_BWD = 6,
  EPI_PEER_RS = 7  // bf16 rows stored straight into their owner rank's reduce-scatter slot (NVLink peer memory)
};

struct GemmArgs {
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
  int splits, k_per_split;  // split-K (fp32 reduce-add output only)
  void* out;
  int64_t ldo;
  int accumulate;
  int split;  // SWIGLU: row offset of W3 inside W13 (= ffn); SWIGLU_BWD: column offset of u in gu (= ffn)
  const void* aux;
  int64_t ld_aux;
  void* out2;
  int64_t ldo2;
  const float* cos_t;
  const float* sin_t;
  int T, hd, rot_cols;
  const int64_t* tgt;
  const float* lse;
  const float* grad_out;
  float* part;    // CE_FWD partials (M, n_blocks, 2)
  float* tlogit;  // CE_FWD target logits (M)
  float alpha;
  void* const* peer;   // PEER_RS: device array of every rank's slot buffer (tp, rows_per_rank, ldo) bf16
  int tp_rank;         // PEER_RS: this rank's slot index in every owner's buffer
  int rows_per_rank;   // PEER_RS: output row r belongs to rank r / rows_per_rank
  const float* scale_a;  // e4m3 operands: inverse tensorwise scales, acc is multiplied by both
  const float* scale_b;  // (NVFP4: the two per-tensor decode scales)
  const uint8_t* sfa;    // block-scaled operands: scale factors of A and B in 512-byte chunks
  const uint8_t* sfb;    // [row tile of 128][chunk along K][32 x 16 bytes]
  int sf_chunks;         // chunks per 128-row tile (k-blocks x chunks per k-block)
  int n_fastest;         // tile order: 1 = consecutive tiles walk N (A blocks reused), 0 = walk M
  int* err;
  // Tensor-parallel all-gather fused into the A loads (bf16, K-major A). A (M x K, row pitch
  // ag_ldd) is this rank's gather buffer of M = ag_tp * rows_per_rank rows; rank q owns rows
  // [q rows_per_rank, (q + 1) rows_per_rank). The kernel's epilogue warps first store this
  // rank's rows (ag_src, pitch ag_lds) into every rank's buffer (ag_dst[p], peer-mapped) in
  // 16-row pieces and count each piece in the flag of its 128-row block on the destination
  // (ag_flags[p][block], red.release.sys); the TMA producer loads an A tile only once this
  // rank's flag of the tile's row block has reached ag_expect (bounded wait, error code 8).
  const void* ag_src;           // nullptr: no fused all-gather
  int64_t ag_lds, ag_ldd;
  void* const* ag_dst;          // device array [ag_tp] of every rank's gather buffer
  uint32_t* const* ag_flags;    // device array [ag_tp] of every rank's flags (one per 128-row block)
  uint32_t ag_expect;           // calls of this gather site so far x kAgPieces
  int ag_tp;
};
// 16-row pieces per 128-row block of a fused all-gather: each adds one to the block's flag.
constexpr int kAgPieces = 8;

// out = op(a) @ op(b); a: (ta ? K x M : M x K) row pitch lda, b: (tb ? N x K : K x N) row pitch ldb.
// The epilogue fields of `g` (out, ldo, accumulate, split, aux, ...) are set by the caller;
// M/N/K, block counts, split-K and err are filled in here. bn = 0 picks the tile width; an
// fp32 output with accumulate=1 (TMA reduce-add) may also be split along K to fill the SMs.
cudaError_t gemm(const void* a, int64_t lda, const void* b, int64_t ldb, bool ta, bool tb, int M, int N, int K,
                 int epi, int bn, GemmArgs g, cudaStream_t st, int splits = 0);
// out = a @ b^T with e4m3 a (M x K) and b (N x K), both row-major (K-major): the only layout of
// the 8-bit GEMM, so the backward passes transposed fp8 copies. g.scale_a / g.scale_b point at
// the operands' inverse tensorwise scales (device floats). Epilogues: BF16, F32 (reduce-add
// with accumulate, split-K allowed), SWIGLU, SWIGLU_BWD, ROPE.
cudaError_t gemm_fp8(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int epi, int bn,
                     GemmArgs g, cudaStream_t st, int splits = 0);
// Tensorwise e4m3 quantization: q = e4m3(sat(x * s)), s = 448 / max(amax|x|, 1e-12), optional
// transposed copy qt (cols x rows), *inv = 1 / s. x is bf16 or fp32 (x_f32), rows x cols with
// row pitch ld; rows and cols multiples of 16. scratch holds fp8_amax_slots() floats.
int fp8_amax_slots();
// Block-scaled GEMM: out = (a @ b^T) with per-block scales applied by the tensor core.
// kind 2 = MXFP8 (e4m3 bytes, ue8m0 scale per 32 along K), kind 3 = NVFP4 (e2m1 packed two per
// byte, ue4m3 scale per 16 along K, g.scale_a / g.scale_b the per-tensor decode scales applied
// in the epilogue). K counts elements; a and b are row-major (K-major) byte matrices; g.sfa /
// g.sfb hold the scales in the chunked layout with cdiv(K, elements per 128 bytes) k-blocks.
// Epilogues: BF16, F32, ROPE, SWIGLU (b rows interleaved 64 of W1, 64 of W3), SWIGLU_BWD.
cudaError_t gemm_bs(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int epi,
                    GemmArgs g, cudaStream_t st, int splits = 0);
// Block-scaled quantization of x (rows x cols, bf16 or fp32) along cols and/or, for x^T, along
// rows: kind 2 MXFP8, kind 3 NVFP4 (g_out: the per-tensor decode scale amax / (6 * 448), from
// scratch partials of fp8_amax pass run here). q: (rows, cols) bytes (NVFP4: cols / 2);
// qt: (cols, rows) (NVFP4: rows / 2); sf / sft: chunked scale layouts. interleave64: the rows
// of x are [W1; W3] of a merged SwiGLU weight and q is written 64 rows of W1, 64 of W3, ...
// stochastic: NVFP4 stochastic rounding with a counter-based generator (seed, element index).
cudaError_t mx_quant(int kind, const void* x, bool x_f32, int rows, int cols, int64_t ld, void* q, void* sf, void* qt,
                     void* sft, float* g_out, float* scratch, bool interleave64, bool stochastic, uint64_t seed,
                     const int64_t* seed_dev, cudaStream_t st);
int64_t mx_sf_bytes(int kind, int rows, int cols);
cudaError_t fp8_quant(const void* x, bool x_f32, int rows, int cols, int64_t ld, void* q, void* qt, float* inv,
                      float* scratch, cudaStream_t st);
int gemm_pick_bn(int M, int N, int epi);
void gemm_plan(int M, int N, int K, int epi, bool can_split, int* bn, int* splits);
int gemm_error_code(bool reset);

// ---------------------------------------------------------------- attention
cudaError_t flash_attn_fwd(const void* qkv, int64_t ld_qkv, void* o, float* lse, int B, int T, int H, int KV, int hd,
                           bool causal, float scale, cudaStream_t st);
// dsum (2*B*H*T floats) and dq_acc (B*T*H*hd floats) are caller-provided scratch.
cudaError_t flash_attn_bwd(const void* dO, const void* qkv, int64_t ld_qkv, const void* o, const float* lse,
                           const float* cos_t, const float* sin_t, void* dqkv, float* dsum, float* dq_acc, int B,
                           int T, int H, int KV, int hd, bool causal, float scale, cudaStream_t st);
int attn_error_code(bool reset);

// ---------------------------------------------------------------- tensor-parallel row collectives
// Over NVLink peer memory (CUDA IPC mappings of every rank's buffers). `dst` / `slots` are
// device arrays of `tp` peer base pointers (this rank's own buffer included).
//   allgather_rows: this rank's rows (rows, d) go to rows [row0, row0 + rows) of every peer's
//                   (N, d) buffer
//   scatter_rows:   rows of a local (N, d) partial go to slot `rank` of their owner's
//                   (tp, N/tp, d) slot buffer
//   sum_slots:      out (n, d) = sum over tp of the local slots (fp32 accumulation)
cudaError_t tp_allgather_rows(const void* src, void* const* dst, int tp, int64_t row0, int64_t rows, int d,
                              cudaStream_t st);
cudaError_t tp_scatter_rows(const void* src, void* const* slots, int tp, int rank, int64_t rows_per_rank, int d,
                            cudaStream_t st);
cudaError_t tp_sum_slots(const void* slots, void* out, int tp, int64_t rows, int d, cudaStream_t st);

// ---------------------------------------------------------------- data-parallel transport
// CUDA-IPC buffers (64-byte handles exchanged by the caller), a flag barrier with bounded
// spins, and the fused reduce-scatter + sharded AdamW + all-gather kernel (comm/dp_fused.cu).
cudaError_t ipc_alloc(size_t bytes, void** ptr, void* handle64);
cudaError_t ipc_open(const void* handle64, void** ptr);
cudaError_t ipc_close(void* ptr);
cudaError_t ipc_free(void* ptr);
cudaError_t dp_barrier(uint32_t* const* pads_dev, uint32_t* my_pad, uint32_t* epoch, int rank, int world, int code,
                       cudaStream_t st);
cudaError_t dp_fused_adamw(float* const* grads_dev, void* const* shadows_dev, float* master, float* m, float* v,
                           int64_t lo, int64_t n, const float* lr, const int* step, AdamHyper h, int world,
                           cudaStream_t st, int max_blocks = 0, bool clear = true);
int dp_error_code(bool reset);
// NVLS data-parallel step (comm/dp_nvls.cu): g_mc / w_mc are the NVLink multicast addresses of
// the flat bf16 gradient and weight buffers; reduce, AdamW on [lo, lo + n), multicast store.
cudaError_t dp_nvls_adamw(const void* g_mc, void* w_mc, float* master, float* m, float* v, int64_t lo, int64_t n,
                          const float* lr, const int* step, AdamHyper h, cudaStream_t st, int max_blocks = 0);

}  // namespace llmt

// PyTorch glue of the llmt native extension (module llmt._C).
//
// The only translation unit that includes torch: it validates tensors (device, dtype,
// layout), allocates outputs through the caching allocator, and calls the plain launch API
// of api.h on the current CUDA stream. Launch errors become Python exceptions.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "api.h"

#define CHECK(cond, ...) TORCH_CHECK(cond, "llmt: ", __VA_ARGS__)
#define CHECK_DT(t, dt) CHECK((t).scalar_type() == (dt), #t " has dtype ", (t).scalar_type(), ", expected ", (dt))

namespace {

cudaStream_t stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

void ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  if (e == cudaErrorInvalidValue && llmt::last_error()[0]) {
    TORCH_CHECK(false, "llmt: ", what, ": ", llmt::last_error());
  }
  TORCH_CHECK(false, "llmt: ", what, ": ", cudaGetErrorString(e));
}

void on_device(const at::Tensor& t, const char* name);

void cuda2d(const at::Tensor& t, const char* name) {
  on_device(t, name);
  CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2D with unit inner stride");
}

// Every pointer a kernel dereferences must be memory of the launching device.
void on_device(const at::Tensor& t, const char* name) {
  CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  CHECK(t.get_device() == c10::cuda::current_device(), name, " is on cuda:", t.get_device(), ", the launch on cuda:",
        (int)c10::cuda::current_device());
}

const void* opt_ptr(const c10::optional<at::Tensor>& t, const char* name = "operand") {
  if (!(t.has_value() && t->defined())) return nullptr;
  on_device(*t, name);
  return t->data_ptr();
}

// ---------------------------------------------------------------- norms
std::vector<at::Tensor> add_rmsnorm_fwd(c10::optional<at::Tensor> a, at::Tensor r, at::Tensor w, double eps,
                                        bool write_s) {
  CHECK(r.is_cuda() && r.is_contiguous(), "r must be a contiguous CUDA tensor");
  on_device(r, "r");
  on_device(w, "w");
  if (a.has_value() && a->defined()) on_device(*a, "a");
  CHECK_DT(r, at::kFloat);
  CHECK_DT(w, at::kFloat);
  const int D = r.size(-1);
  const int64_t N = r.numel() / D;
  CHECK(w.numel() == D && w.is_contiguous(), "w must be contiguous with ", D, " elements");
  const bool has_a = a.has_value() && a->defined();
  if (has_a) {
    CHECK_DT((*a), at::kBFloat16);
    CHECK(a->is_contiguous() && a->numel() == r.numel(), "a must be contiguous and match r");
  }
  auto y = at::empty(r.sizes(), r.options().dtype(at::kBFloat16));
  auto rstd = at::empty({N}, r.options());
  at::Tensor s;
  if (write_s) s = at::empty_like(r);
  ok(llmt::add_rmsnorm_fwd(has_a ? a->data_ptr() : nullptr, r.data_ptr<float>(), w.data_ptr<float>(), y.data_ptr(),
                           write_s ? s.data_ptr<float>() : nullptr, rstd.data_ptr<float>(), N, D, (float)eps, stream()),
     "add_rmsnorm_fwd");
  return {y, s, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor s, at::Tensor w, at::Tensor rstd,
                                    c10::optional<at::Tensor> ds_in, at::Tensor dw, at::Tensor ticket,
                                    bool write_ds16, bool accumulate) {
  CHECK_DT(dy, at::kBFloat16);
  CHECK_DT(s, at::kFloat);
  CHECK_DT(dw, at::kFloat);
  CHECK_DT(ticket, at::kInt);
  for (auto* t : {&dy, &s, &w, &rstd, &dw}) on_device(*t, "rmsnorm_bwd operand");
  if (ds_in.has_value() && ds_in->defined()) on_device(*ds_in, "ds_in");
  CHECK(dy.is_contiguous() && s.is_contiguous() && dy.numel() == s.numel(), "dy/s must be contiguous and match");
  const int D = s.size(-1);
  const int64_t N = s.numel() / D;
  CHECK(dw.numel() == D && dw.is_contiguous(), "dw must be contiguous with ", D, " elements");
  const bool has_dsin = ds_in.has_value() && ds_in->defined();
  if (has_dsin) {
    CHECK_DT((*ds_in), at::kFloat);
    CHECK(ds_in->is_contiguous() && ds_in->numel() == s.numel(), "ds_in must be contiguous and match s");
  }
  auto ds = at::empty_like(s);
  at::Tensor ds16;
  if (write_ds16) ds16 = at::empty(s.sizes(), s.options().dtype(at::kBFloat16));
  auto part = at::empty({llmt::rmsnorm_bwd_partials(N, D), D}, s.options());
  ok(llmt::rmsnorm_bwd(dy.data_ptr(), s.data_ptr<float>(), w.data_ptr<float>(), rstd.data_ptr<float>(),
                       has_dsin ? ds_in->data_ptr<float>() : nullptr, ds.data_ptr<float>(),
                       write_ds16 ? ds16.data_ptr() : nullptr, part.data_ptr<float>(), dw.data_ptr<float>(),
                       reinterpret_cast<unsigned*>(ticket.data_ptr<int>()), N, D, accumulate ? 1 : 0, stream()),
     "rmsnorm_bwd");
  return {ds, ds16};
}

// ---------------------------------------------------------------- elementwise
void swiglu_fwd(at::Tensor g, at::Tensor u, at::Tensor h) {
  cuda2d(g, "g");
  cuda2d(u, "u");
  cuda2d(h, "h");
  CHECK(g.stride(0) == u.stride(0), "g and u must share a row stride");
  CHECK_DT(g, at::kBFloat16);
  ok(llmt::swiglu_fwd(g.data_ptr(), u.data_ptr(), g.stride(0), h.data_ptr(), h.stride(0), g.size(0), g.size(1),
                      stream()),
     "swiglu_fwd");
}

void swiglu_bwd(at::Tensor dh, at::Tensor g, at::Tensor u, at::Tensor dg, at::Tensor du) {
  for (auto* t : {&dh, &g, &u, &dg, &du}) cuda2d(*t, "swiglu operand");
  CHECK(g.stride(0) == u.stride(0) && dg.stride(0) == du.stride(0), "paired row strides differ");
  ok(llmt::swiglu_bwd(dh.data_ptr(), dh.stride(0), g.data_ptr(), u.data_ptr(), g.stride(0), dg.data_ptr(),
                      du.data_ptr(), dg.stride(0), g.size(0), g.size(1), stream()),
     "swiglu_bwd");
}

void rope_inplace(at::Tensor qkv, at::Tensor cos_t, at::Tensor sin_t, int64_t T, int64_t n_rot_heads, int64_t hd,
                  bool backward) {
  CHECK_DT(qkv, at::kBFloat16);
  CHECK_DT(cos_t, at::kFloat);
  for (auto* t : {&qkv, &cos_t, &sin_t}) on_device(*t, "rope operand");
  CHECK(qkv.is_contiguous() && cos_t.is_contiguous() && sin_t.is_contiguous(), "rope operands must be contiguous");
  CHECK(cos_t.size(0) >= T && cos_t.size(1) == hd, "rope table too small");
  const int64_t ld = qkv.size(-1);
  ok(llmt::rope_inplace(qkv.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), qkv.numel() / ld, (int)T,
                        (int)n_rot_heads, (int)hd, ld, backward, stream()),
     "rope_inplace");
}

void embedding_fwd(at::Tensor idx, at::Tensor W, at::Tensor x, c10::optional<at::Tensor> err, int64_t v0,
                   bool partial) {
  CHECK_DT(idx, at::kLong);
  CHECK_DT(W, at::kFloat);
  for (auto* t : {&idx, &W, &x}) on_device(*t, "embedding operand");
  CHECK(idx.is_contiguous() && W.is_contiguous() && x.is_contiguous(), "embedding operands must be contiguous");
  ok(llmt::embedding_fwd(idx.data_ptr<int64_t>(), W.data_ptr<float>(), x.data_ptr<float>(), idx.numel(), W.size(1),
                         W.size(0), v0, partial, err.has_value() && err->defined() ? err->data_ptr<int>() : nullptr,
                         stream()),
     "embedding_fwd");
}

void embedding_bwd(at::Tensor idx, at::Tensor dx, at::Tensor dW, int64_t v0) {
  CHECK_DT(dx, at::kFloat);
  CHECK_DT(dW, at::kFloat);
  for (auto* t : {&idx, &dx, &dW}) on_device(*t, "embedding operand");
  CHECK(idx.is_contiguous() && dx.is_contiguous() && dW.is_contiguous(), "embedding grads must be contiguous");
  ok(llmt::embedding_bwd(idx.data_ptr<int64_t>(), dx.data_ptr<float>(), dW.data_ptr<float>(), idx.numel(), dW.size(1),
                         dW.size(0), v0, stream()),
     "embedding_bwd");
}

// ---------------------------------------------------------------- optimizer
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p16, at::Tensor lr,
                at::Tensor step, double b1, double b2, double eps, double wd, double grad_scale, bool zero_grad,
                int64_t max_blocks) {
  for (auto* t : {&p, &g, &m, &v, &lr, &step}) on_device(*t, "adamw operand");
  for (auto* t : {&p, &g, &m, &v}) {
    CHECK_DT((*t), at::kFloat);
    CHECK(t->is_contiguous() && t->numel() == p.numel(), "adamw buffers must be contiguous and equal-sized");
  }
  CHECK_DT(lr, at::kFloat);
  CHECK_DT(step, at::kInt);
  void* p16p = nullptr;
  if (p16.has_value() && p16->defined()) {
    CHECK_DT((*p16), at::kBFloat16);
    CHECK(p16->numel() == p.numel() && p16->is_contiguous(), "adamw: bf16 copy size mismatch");
    p16p = p16->data_ptr();
  }
  llmt::AdamHyper h{(float)b1, (float)b2, (float)eps, (float)wd, (float)grad_scale};
  ok(llmt::adamw_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), p16p,
                      p.numel(), lr.data_ptr<float>(), step.data_ptr<int>(), h, zero_grad, stream(), (int)max_blocks),
     "adamw_step");
}

void cast_bf16(at::Tensor x, at::Tensor y, int64_t max_blocks) {
  CHECK_DT(x, at::kFloat);
  CHECK_DT(y, at::kBFloat16);
  on_device(x, "x");
  on_device(y, "y");
  CHECK(x.numel() == y.numel() && x.is_contiguous() && y.is_contiguous(), "cast_bf16: bad args");
  ok(llmt::cast_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), stream(), (int)max_blocks), "cast_bf16");
}

// ---------------------------------------------------------------- cross entropy
void ce_fwd_rows(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor loss) {
  cuda2d(logits, "logits");
  CHECK_DT(logits, at::kBFloat16);
  CHECK_DT(targets, at::kLong);
  ok(llmt::ce_fwd_rows(logits.data_ptr(), logits.stride(0), targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
                       loss.data_ptr<float>(), logits.size(0), logits.size(1), stream()),
     "ce_fwd_rows");
}

void ce_bwd_rows(at::Tensor logits, at::Tensor targets, at::Tensor lse, c10::optional<at::Tensor> grad_out,
                 double scale) {
  cuda2d(logits, "logits");
  CHECK_DT(logits, at::kBFloat16);
  ok(llmt::ce_bwd_rows(logits.data_ptr(), logits.stride(0), targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
                       static_cast<const float*>(opt_ptr(grad_out, "grad_out")), (float)scale, logits.size(0), logits.size(1),
                       stream()),
     "ce_bwd_rows");
}

void ce_combine(at::Tensor part, at::Tensor tlogit, at::Tensor tgt, at::Tensor lse, at::Tensor loss, int64_t nblk,
                int64_t V) {
  for (auto* t : {&part, &tlogit, &tgt, &lse, &loss}) on_device(*t, "ce_combine operand");
  ok(llmt::ce_combine(part.data_ptr<float>(), tlogit.data_ptr<float>(), tgt.data_ptr<int64_t>(), lse.data_ptr<float>(),
                      loss.data_ptr<float>(), (int)lse.numel(), (int)nblk, (int)V, stream()),
     "ce_combine");
}

// ---------------------------------------------------------------- fp8 quantization
void fp8_quant(at::Tensor x, at::Tensor q, c10::optional<at::Tensor> qt, at::Tensor inv, at::Tensor scratch) {
  cuda2d(x, "x");
  CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "fp8_quant: x must be bf16 or fp32");
  CHECK(x.stride(1) == 1, "fp8_quant: x rows must be contiguous");
  const int64_t rows = x.size(0), cols = x.size(1);
  on_device(q, "q");
  CHECK_DT(q, at::kFloat8_e4m3fn);
  CHECK(q.is_contiguous() && q.numel() == rows * cols, "fp8_quant: q must be a contiguous rows x cols tensor");
  void* qtp = nullptr;
  if (qt.has_value() && qt->defined()) {
    on_device(*qt, "qt");
    CHECK_DT((*qt), at::kFloat8_e4m3fn);
    CHECK(qt->is_contiguous() && qt->numel() == rows * cols, "fp8_quant: qt must be a contiguous cols x rows tensor");
    qtp = qt->data_ptr();
  }
  for (auto* t : {&inv, &scratch}) {
    on_device(*t, "fp8_quant scale buffer");
    CHECK_DT((*t), at::kFloat);
  }
  CHECK(scratch.numel() >= llmt::fp8_amax_slots(), "fp8_quant: scratch needs fp8_amax_slots() floats");
  ok(llmt::fp8_quant(x.data_ptr(), x.scalar_type() == at::kFloat, (int)rows, (int)cols, x.stride(0), q.data_ptr(), qtp,
                     inv.data_ptr<float>(), scratch.data_ptr<float>(), stream()),
     "fp8_quant");
}

void mx_quant(int64_t kind, at::Tensor x, c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf,
              c10::optional<at::Tensor> qt, c10::optional<at::Tensor> sft, c10::optional<at::Tensor> g,
              c10::optional<at::Tensor> scratch, bool interleave64, bool stochastic, int64_t seed,
              c10::optional<at::Tensor> seed_dev) {
  cuda2d(x, "x");
  CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "mx_quant: x must be bf16 or fp32");
  const int64_t rows = x.size(0), cols = x.size(1);
  const int64_t per = kind == 3 ? 2 : 1;
  auto bytes = [&](c10::optional<at::Tensor>& t, int64_t n, const char* name) -> void* {
    if (!t.has_value() || !t->defined()) return nullptr;
    on_device(*t, name);
    CHECK(t->element_size() == 1 && t->is_contiguous() && t->numel() >= n, name, ": contiguous bytes, at least ", n);
    return t->data_ptr();
  };
  void* qp = bytes(q, rows * cols / per, "q");
  void* qtp = bytes(qt, rows * cols / per, "qt");
  void* sfp = bytes(sf, qp ? llmt::mx_sf_bytes((int)kind, rows, cols) : 0, "sf");
  void* sftp = bytes(sft, qtp ? llmt::mx_sf_bytes((int)kind, cols, rows) : 0, "sft");
  float* gp = nullptr;
  float* sp = nullptr;
  if (kind == 3) {
    CHECK(g.has_value() && scratch.has_value(), "mx_quant: NVFP4 needs g and scratch");
    for (auto* t : {&*g, &*scratch}) {
      on_device(*t, "mx_quant scale buffer");
      CHECK_DT((*t), at::kFloat);
    }
    CHECK(scratch->numel() >= llmt::fp8_amax_slots(), "mx_quant: scratch too small");
    gp = g->data_ptr<float>();
    sp = scratch->data_ptr<float>();
  }
  ok(llmt::mx_quant((int)kind, x.data_ptr(), x.scalar_type() == at::kFloat, (int)rows, (int)cols, x.stride(0), qp, sfp, qtp,
                    sftp, gp, sp, interleave64, stochastic, (uint64_t)seed,
                    static_cast<const int64_t*>(opt_ptr(seed_dev, "seed_dev")), stream()),
     "mx_quant");
}

// ---------------------------------------------------------------- GEMM
void gemm(at::Tensor a, at::Tensor b, bool ta, bool tb, int64_t epi, at::Tensor out, bool accumulate,
          c10::optional<at::Tensor> aux, c10::optional<at::Tensor> out2, int64_t split, c10::optional<at::Tensor> cos_t,
          c10::optional<at::Tensor> sin_t, int64_t T, int64_t hd, int64_t rot_cols, c10::optional<at::Tensor> tgt,
          c10::optional<at::Tensor> lse, c10::optional<at::Tensor> grad_out, c10::optional<at::Tensor> part,
          c10::optional<at::Tensor> tlogit, double alpha, int64_t bn, int64_t splits, c10::optional<at::Tensor> peer,
          int64_t tp_rank, int64_t rows_per_rank, c10::optional<at::Tensor> scale_a, c10::optional<at::Tensor> scale_b,
          int64_t kind, c10::optional<at::Tensor> sfa, c10::optional<at::Tensor> sfb, c10::optional<at::Tensor> ag_src,
          c10::optional<at::Tensor> ag_dst, c10::optional<at::Tensor> ag_flags, int64_t ag_expect, int64_t ag_tp) {
  cuda2d(a, "a");
  cuda2d(b, "b");
  const bool bs = kind == 2 || kind == 3;
  const bool f8 = !bs && a.scalar_type() == at::kFloat8_e4m3fn;
  CHECK(kind == 0 || bs, "gemm: kind must be 0 (by dtype), 2 (MXFP8) or 3 (NVFP4)");
  if (bs) {
    CHECK(!ta && tb, "block-scaled gemm: both operands K-major (a: M x K, b: N x K)");
    CHECK(a.element_size() == 1 && b.element_size() == 1, "block-scaled gemm: byte operands");
    CHECK(sfa.has_value() && sfb.has_value(), "block-scaled gemm needs sfa and sfb");
    for (auto* t : {&*sfa, &*sfb}) {
      on_device(*t, "scale factors");
      CHECK(t->element_size() == 1 && t->is_contiguous(), "scale factors: contiguous bytes");
    }
    if (kind == 3) {
      CHECK(scale_a.has_value() && scale_b.has_value(), "NVFP4 gemm needs the decode scales");
      for (auto* t : {&*scale_a, &*scale_b}) {
        on_device(*t, "decode scale");
        CHECK_DT((*t), at::kFloat);
      }
    }
  } else if (f8) {
    CHECK_DT(b, at::kFloat8_e4m3fn);
    CHECK(!ta && tb, "fp8 gemm: both operands K-major (a: M x K, b: N x K)");
    CHECK(scale_a.has_value() && scale_b.has_value(), "fp8 gemm needs scale_a and scale_b");
    for (auto* t : {&*scale_a, &*scale_b}) {
      on_device(*t, "fp8 scale");
      CHECK_DT((*t), at::kFloat);
    }
  } else {
    CHECK_DT(a, at::kBFloat16);
    CHECK_DT(b, at::kBFloat16);
  }
  on_device(out, "out");
  const int kmul = kind == 3 ? 2 : 1;  // NVFP4 bytes hold two elements
  const int M = ta ? a.size(1) : a.size(0);
  const int K = (ta ? a.size(0) : a.size(1)) * kmul;
  int N = tb ? b.size(0) : b.size(1);
  const int Kb = (tb ? b.size(1) : b.size(0)) * kmul;
  CHECK(K == Kb, "gemm inner dims differ: ", K, " vs ", Kb);
  if (epi == llmt::EPI_SWIGLU) {
    CHECK(tb && b.size(0) == 2 * split, "SWIGLU gemm: b must be W13 (2*ffn, K)");
    N = (int)split;
  }
  switch (epi) {
    case llmt::EPI_BF16: case llmt::EPI_ROPE: case llmt::EPI_CE_BWD: case llmt::EPI_SWIGLU:
      CHECK_DT(out, at::kBFloat16);
      CHECK(out.dim() == 2 && out.size(0) >= M && out.size(1) >= N && out.stride(1) == 1 && out.stride(0) % 8 == 0,
            "gemm: bf16 output must be (M, N) row-major with a 16-byte-multiple pitch");
      break;
    case llmt::EPI_F32:
      CHECK_DT(out, at::kFloat);
      CHECK(out.dim() == 2 && out.size(0) >= M && out.size(1) >= N && out.stride(1) == 1 && out.stride(0) % 4 == 0,
            "gemm: fp32 output must be (M, N) row-major with a 16-byte-multiple pitch");
      break;
    case llmt::EPI_SWIGLU_BWD: case llmt::EPI_CE_FWD: break;
    case llmt::EPI_PEER_RS:
      CHECK(peer.has_value() && peer->defined() && peer->scalar_type() == at::kLong, "PEER_RS gemm needs peer slots");
      CHECK(out.dim() == 2 && out.size(1) == N && out.is_contiguous(), "PEER_RS: out is this rank's slot buffer (., N)");
      break;
    default: CHECK(false, "gemm: unknown epilogue ", epi);
  }
  llmt::GemmArgs g{};
  g.out = out.data_ptr();
  g.ldo = out.dim() == 2 ? out.stride(0) : N;
  g.accumulate = accumulate ? 1 : 0;
  g.split = (int)split;
  g.alpha = (float)alpha;
  if (aux.has_value() && aux->defined()) {
    on_device(*aux, "aux");
    CHECK_DT((*aux), at::kBFloat16);
    g.aux = aux->data_ptr();
    g.ld_aux = aux->stride(0);
  }
  if (out2.has_value() && out2->defined()) {
    on_device(*out2, "out2");
    CHECK_DT((*out2), at::kBFloat16);
    g.out2 = out2->data_ptr();
    g.ldo2 = out2->stride(0);
  }
  g.cos_t = static_cast<const float*>(opt_ptr(cos_t, "cos_t"));
  g.sin_t = static_cast<const float*>(opt_ptr(sin_t, "sin_t"));
  g.T = (int)T;
  g.hd = (int)hd;
  g.rot_cols = (int)rot_cols;
  g.tgt = static_cast<const int64_t*>(opt_ptr(tgt, "tgt"));
  g.lse = static_cast<const float*>(opt_ptr(lse, "lse"));
  g.grad_out = static_cast<const float*>(opt_ptr(grad_out, "grad_out"));
  g.part = static_cast<float*>(const_cast<void*>(opt_ptr(part, "part")));
  g.tlogit = static_cast<float*>(const_cast<void*>(opt_ptr(tlogit, "tlogit")));
  g.peer = reinterpret_cast<void* const*>(const_cast<void*>(opt_ptr(peer, "peer")));
  g.tp_rank = (int)tp_rank;
  g.rows_per_rank = (int)rows_per_rank;
  if (ag_src.has_value() && ag_src->defined()) {
    // fused all-gather: this rank's rows (rows_per_rank, K) bf16; a is this rank's gather buffer
    cuda2d(*ag_src, "ag_src");
    CHECK(kind == 0 && !f8, "fused all-gather: bf16 operands only");
    CHECK_DT((*ag_src), at::kBFloat16);
    CHECK(!ta && ag_src->size(0) == rows_per_rank && ag_src->size(1) == a.size(1) && ag_src->stride(1) == 1,
          "ag_src must be this rank's (rows_per_rank, K) rows of a row-major A");
    CHECK(ag_dst.has_value() && ag_flags.has_value() && ag_dst->scalar_type() == at::kLong &&
              ag_flags->scalar_type() == at::kLong && ag_dst->numel() == ag_tp && ag_flags->numel() == ag_tp,
          "fused all-gather needs ag_dst and ag_flags: int64 device arrays of ag_tp pointers");
    on_device(*ag_dst, "ag_dst");
    on_device(*ag_flags, "ag_flags");
    g.ag_src = ag_src->data_ptr();
    g.ag_lds = ag_src->stride(0);
    g.ag_dst = reinterpret_cast<void* const*>(ag_dst->data_ptr());
    g.ag_flags = reinterpret_cast<uint32_t* const*>(ag_flags->data_ptr());
    g.ag_expect = (uint32_t)ag_expect;
    g.ag_tp = (int)ag_tp;
  }
  if (epi == llmt::EPI_ROPE) CHECK(g.cos_t && g.sin_t && T > 0, "ROPE gemm needs rope tables and T");
  if (epi == llmt::EPI_SWIGLU) CHECK(g.aux && aux->stride(0) % 8 == 0, "SWIGLU gemm needs the gu save buffer");
  if (epi == llmt::EPI_SWIGLU_BWD) CHECK(g.aux && g.out2 && split == N, "SWIGLU_BWD gemm args");
  if (epi == llmt::EPI_CE_FWD) {
    CHECK(g.tgt && g.part && g.tlogit, "CE_FWD gemm args");
    const int BN = bn ? (int)bn : llmt::gemm_pick_bn(M, N, (int)epi);
    CHECK(part->numel() >= (int64_t)M * ((N + BN - 1) / BN) * 2, "CE_FWD partial buffer too small");
  }
  if (epi == llmt::EPI_CE_BWD) CHECK(g.tgt && g.lse, "CE_BWD gemm args");
  if (bs) {
    if (kind == 3) {
      g.scale_a = scale_a->data_ptr<float>();
      g.scale_b = scale_b->data_ptr<float>();
    }
    g.sfa = static_cast<const uint8_t*>(sfa->data_ptr());
    g.sfb = static_cast<const uint8_t*>(sfb->data_ptr());
    const int kbytes = K / kmul;
    const int64_t need_a = llmt::mx_sf_bytes((int)kind, M, K), need_b = llmt::mx_sf_bytes((int)kind, b.size(0), K);
    CHECK(sfa->numel() >= need_a && sfb->numel() >= need_b, "block-scaled gemm: scale buffers too small");
    (void)kbytes;
    ok(llmt::gemm_bs((int)kind, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), M, N, K, (int)epi, g, stream(),
                     (int)splits),
       "gemm_bs");
    return;
  }
  if (f8) {
    g.scale_a = scale_a->data_ptr<float>();
    g.scale_b = scale_b->data_ptr<float>();
    ok(llmt::gemm_fp8(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), M, N, K, (int)epi, (int)bn, g, stream(),
                      (int)splits),
       "gemm_fp8");
    return;
  }
  ok(llmt::gemm(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), ta, tb, M, N, K, (int)epi, (int)bn, g, stream(),
                (int)splits),
     "gemm");
}

// ---------------------------------------------------------------- attention
std::vector<at::Tensor> flash_attn_fwd(at::Tensor qkv, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd,
                                       bool causal, double scale) {
  cuda2d(qkv, "qkv");
  CHECK_DT(qkv, at::kBFloat16);
  CHECK(qkv.size(0) == B * T && qkv.size(1) >= (H + 2 * KV) * hd, "flash_attn_fwd: qkv shape mismatch");
  auto o = at::empty({B * T, H * hd}, qkv.options());
  auto lse = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  ok(llmt::flash_attn_fwd(qkv.data_ptr(), qkv.stride(0), o.data_ptr(), lse.data_ptr<float>(), (int)B, (int)T, (int)H,
                          (int)KV, (int)hd, causal, (float)scale, stream()),
     "flash_attn_fwd");
  return {o, lse};
}

at::Tensor flash_attn_bwd(at::Tensor dO, at::Tensor qkv, at::Tensor o, at::Tensor lse, at::Tensor cos_t,
                          at::Tensor sin_t, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd, bool causal,
                          double scale) {
  CHECK_DT(dO, at::kBFloat16);
  CHECK_DT(qkv, at::kBFloat16);
  CHECK_DT(o, at::kBFloat16);
  CHECK_DT(lse, at::kFloat);
  for (auto* t : {&dO, &qkv, &o, &lse, &cos_t, &sin_t}) on_device(*t, "flash_attn_bwd operand");
  CHECK(dO.is_contiguous() && o.is_contiguous() && qkv.is_contiguous() && lse.is_contiguous(),
        "flash_attn_bwd: operands must be contiguous");
  CHECK(dO.numel() == B * T * H * hd && o.numel() == dO.numel(), "flash_attn_bwd: dO/o shape");
  CHECK(qkv.size(0) == B * T && qkv.size(1) == (H + 2 * KV) * hd, "flash_attn_bwd: qkv shape");
  CHECK(cos_t.size(0) >= T && cos_t.size(1) == hd && cos_t.is_contiguous() && sin_t.is_contiguous(),
        "flash_attn_bwd: rope tables");
  auto dqkv = at::empty_like(qkv);
  auto dsum = at::empty({2, B, H, T}, lse.options());
  auto dq_acc = at::empty({B * T, H * hd}, lse.options());
  ok(llmt::flash_attn_bwd(dO.data_ptr(), qkv.data_ptr(), qkv.stride(0), o.data_ptr(), lse.data_ptr<float>(),
                          cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), dqkv.data_ptr(), dsum.data_ptr<float>(),
                          dq_acc.data_ptr<float>(), (int)B, (int)T, (int)H, (int)KV, (int)hd, causal, (float)scale,
                          stream()),
     "flash_attn_bwd");
  return dqkv;
}

// ---------------------------------------------------------------- data-parallel transport
pybind11::tuple ipc_alloc(int64_t bytes) {
  void* ptr = nullptr;
  char h[64];
  ok(llmt::ipc_alloc((size_t)bytes, &ptr, h), "ipc_alloc");
  return pybind11::make_tuple((int64_t)reinterpret_cast<uintptr_t>(ptr), pybind11::bytes(h, 64));
}

int64_t ipc_open(pybind11::bytes handle) {
  std::string h = handle;
  CHECK(h.size() == 64, "ipc handle must be 64 bytes");
  void* ptr = nullptr;
  ok(llmt::ipc_open(h.data(), &ptr), "ipc_open");
  return (int64_t)reinterpret_cast<uintptr_t>(ptr);
}

void ipc_close(int64_t ptr) { ok(llmt::ipc_close(reinterpret_cast<void*>(ptr)), "ipc_close"); }
void ipc_free(int64_t ptr) { ok(llmt::ipc_free(reinterpret_cast<void*>(ptr)), "ipc_free"); }

// Non-owning tensor over device memory this library allocated (the Python owner frees it).
at::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel},
                       at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, (int)device)));
}

void dp_barrier(at::Tensor pads_dev, int64_t my_pad, at::Tensor epoch, int64_t rank, int64_t world, int64_t code) {
  CHECK_DT(pads_dev, at::kLong);
  CHECK_DT(epoch, at::kInt);
  ok(llmt::dp_barrier(reinterpret_cast<uint32_t* const*>(pads_dev.data_ptr<int64_t>()),
                      reinterpret_cast<uint32_t*>(my_pad), reinterpret_cast<uint32_t*>(epoch.data_ptr<int>()),
                      (int)rank, (int)world, (int)code, stream()),
     "dp_barrier");
}

void dp_fused_adamw(at::Tensor grads_dev, at::Tensor shadows_dev, at::Tensor master, at::Tensor m, at::Tensor v,
                    int64_t lo, int64_t n, at::Tensor lr, at::Tensor step, double b1, double b2, double eps, double wd,
                    double grad_scale, int64_t world, int64_t max_blocks, bool clear) {
  CHECK_DT(grads_dev, at::kLong);
  CHECK_DT(shadows_dev, at::kLong);
  CHECK(grads_dev.numel() == world && shadows_dev.numel() == world, "peer pointer arrays must have world entries");
  CHECK(m.numel() >= n && v.numel() >= n && master.numel() >= lo + n, "shard bounds exceed the buffers");
  llmt::AdamHyper h{(float)b1, (float)b2, (float)eps, (float)wd, (float)grad_scale};
  ok(llmt::dp_fused_adamw(reinterpret_cast<float* const*>(grads_dev.data_ptr<int64_t>()),
                          reinterpret_cast<void* const*>(shadows_dev.data_ptr<int64_t>()), master.data_ptr<float>(),
                          m.data_ptr<float>(), v.data_ptr<float>(), lo, n, lr.data_ptr<float>(), step.data_ptr<int>(),
                          h, (int)world, stream(), (int)max_blocks, clear),
     "dp_fused_adamw");
}

void dp_nvls_adamw(int64_t g_mc, int64_t w_mc, at::Tensor master, at::Tensor m, at::Tensor v, int64_t lo, int64_t n,
                   at::Tensor lr, at::Tensor step, double b1, double b2, double eps, double wd, double grad_scale,
                   int64_t max_blocks) {
  on_device(master, "master");
  on_device(m, "m");
  on_device(v, "v");
  CHECK(g_mc != 0 && w_mc != 0, "dp_nvls_adamw: multicast addresses are null (no NVLS support)");
  CHECK(m.numel() >= n && v.numel() >= n && master.numel() >= lo + n, "shard bounds exceed the buffers");
  llmt::AdamHyper h{(float)b1, (float)b2, (float)eps, (float)wd, (float)grad_scale};
  ok(llmt::dp_nvls_adamw(reinterpret_cast<const void*>(g_mc), reinterpret_cast<void*>(w_mc), master.data_ptr<float>(),
                         m.data_ptr<float>(), v.data_ptr<float>(), lo, n, lr.data_ptr<float>(), step.data_ptr<int>(), h,
                         stream(), (int)max_blocks),
     "dp_nvls_adamw");
}

#ifdef LLMT_DEBUG_BOUNDS
// Self-test of the bounds-checked build: a store at index `i` of an n-float buffer, guarded by
// LLMT_IN. With i >= n the guard records the site and skips the store (nothing is written out
// of bounds); the record is read back with bounds_error(). Only this build has it.
void bounds_probe(at::Tensor buf, int64_t i) {
  on_device(buf, "buf");
  CHECK_DT(buf, at::kFloat);
  ok(llmt::bounds_probe(buf.data_ptr<float>(), buf.numel(), i, stream()), "bounds_probe");
}
#endif

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  using namespace pybind11::literals;
  m.doc() = "llmt native sm_100a kernels";
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd, "a"_a, "r"_a, "w"_a, "eps"_a, "write_s"_a);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, "dy"_a, "s"_a, "w"_a, "rstd"_a, "ds_in"_a, "dw"_a, "ticket"_a, "write_ds16"_a,
        "accumulate"_a);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_inplace", &rope_inplace);
  m.def("embedding_fwd", &embedding_fwd, "idx"_a, "W"_a, "x"_a, "err"_a = py::none(), "v0"_a = 0,
        "partial"_a = false);
  m.def("embedding_bwd", &embedding_bwd, "idx"_a, "dx"_a, "dW"_a, "v0"_a = 0);
  m.def("adamw_step", &adamw_step, "p"_a, "g"_a, "m"_a, "v"_a, "p16"_a, "lr"_a, "step"_a, "b1"_a, "b2"_a, "eps"_a,
        "wd"_a, "grad_scale"_a, "zero_grad"_a = false, "max_blocks"_a = 0);
  m.def("cast_bf16", &cast_bf16, "x"_a, "y"_a, "max_blocks"_a = 0);
  m.def("ce_fwd_rows", &ce_fwd_rows);
  m.def("ce_bwd_rows", &ce_bwd_rows);
  m.def("ce_combine", &ce_combine);
  m.def("gemm", &gemm, "a"_a, "b"_a, "ta"_a, "tb"_a, "epi"_a, "out"_a, "accumulate"_a = false, "aux"_a = py::none(),
        "out2"_a = py::none(), "split"_a = 0, "cos_t"_a = py::none(), "sin_t"_a = py::none(), "T"_a = 0, "hd"_a = 0,
        "rot_cols"_a = 0, "tgt"_a = py::none(), "lse"_a = py::none(), "grad_out"_a = py::none(), "part"_a = py::none(),
        "tlogit"_a = py::none(), "alpha"_a = 1.0, "bn"_a = 0, "splits"_a = 0, "peer"_a = py::none(), "tp_rank"_a = 0, "rows_per_rank"_a = 0,
        "scale_a"_a = py::none(), "scale_b"_a = py::none(), "kind"_a = 0, "sfa"_a = py::none(), "sfb"_a = py::none(),
        "ag_src"_a = py::none(), "ag_dst"_a = py::none(), "ag_flags"_a = py::none(), "ag_expect"_a = 0, "ag_tp"_a = 0);
  m.def("mx_sf_bytes", &llmt::mx_sf_bytes);
  m.def("mx_quant", &mx_quant, "kind"_a, "x"_a, "q"_a, "sf"_a, "qt"_a, "sft"_a, "g"_a, "scratch"_a,
        "interleave64"_a = false, "stochastic"_a = false, "seed"_a = 0, "seed_dev"_a = py::none());
  m.def("fp8_amax_slots", &llmt::fp8_amax_slots);
  m.def("fp8_quant", &fp8_quant, "x"_a, "q"_a, "qt"_a, "inv"_a, "scratch"_a);
  m.def("gemm_error_code", &llmt::gemm_error_code, "reset"_a = false);
  m.def("gemm_plan", [](int64_t M, int64_t N, int64_t K, int64_t epi, bool can_split) {
    int bn = 0, splits = 1;
    llmt::gemm_plan((int)M, (int)N, (int)K, (int)epi, can_split, &bn, &splits);
    return std::make_tuple(bn, splits);
  });
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("attn_error_code", &llmt::attn_error_code, "reset"_a = false);
  m.def("set_reserved_sms", &llmt::set_reserved_sms, "n"_a);
  m.def("reserved_sms", &llmt::reserved_sms);
  m.def("tp_allgather_rows", [](at::Tensor src, at::Tensor dst, int64_t tp, int64_t row0) {
    on_device(src, "src");
    CHECK(src.is_contiguous() && src.scalar_type() == at::kBFloat16 && src.dim() == 2, "tp_allgather_rows: src");
    ok(llmt::tp_allgather_rows(src.data_ptr(), reinterpret_cast<void* const*>(dst.data_ptr<int64_t>()), (int)tp, row0,
                               src.size(0), (int)src.size(1), stream()),
       "tp_allgather_rows");
  });
  m.def("tp_scatter_rows", [](at::Tensor src, at::Tensor slots, int64_t tp, int64_t rank) {
    on_device(src, "src");
    CHECK(src.is_contiguous() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.size(0) % tp == 0,
          "tp_scatter_rows: src");
    ok(llmt::tp_scatter_rows(src.data_ptr(), reinterpret_cast<void* const*>(slots.data_ptr<int64_t>()), (int)tp,
                             (int)rank, src.size(0) / tp, (int)src.size(1), stream()),
       "tp_scatter_rows");
  });
  m.def("tp_sum_slots", [](at::Tensor slots, at::Tensor out, int64_t tp) {
    on_device(slots, "slots");
    on_device(out, "out");
    CHECK(out.is_contiguous() && slots.is_contiguous() && slots.numel() == tp * out.numel(), "tp_sum_slots: shapes");
    ok(llmt::tp_sum_slots(slots.data_ptr(), out.data_ptr(), (int)tp, out.size(0), (int)out.size(1), stream()),
       "tp_sum_slots");
  });
  m.def("sm_count", &llmt::sm_count);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("dp_barrier", &dp_barrier);
  m.def("dp_fused_adamw", &dp_fused_adamw, "grads_dev"_a, "shadows_dev"_a, "master"_a, "m"_a, "v"_a, "lo"_a, "n"_a,
        "lr"_a, "step"_a, "b1"_a, "b2"_a, "eps"_a, "wd"_a, "grad_scale"_a, "world"_a, "max_blocks"_a = 0,
        "clear"_a = true);
  m.def("dp_error_code", &llmt::dp_error_code, "reset"_a = false);
  m.def("bounds_error", &llmt::bounds_error, "reset"_a = false);
  m.def("bounds_checking", &llmt::bounds_checking);
#ifdef LLMT_DEBUG_BOUNDS
  m.def("bounds_probe", &bounds_probe, "buf"_a, "i"_a);
#endif
  m.def("dp_nvls_adamw", &dp_nvls_adamw, "g_mc"_a, "w_mc"_a, "master"_a, "m"_a, "v"_a, "lo"_a, "n"_a, "lr"_a, "step"_a,
        "b1"_a, "b2"_a, "eps"_a, "wd"_a, "grad_scale"_a, "max_blocks"_a = 0);
}

// Python bindings of the llmt native extension (one module, llmt._C).
#include <torch/extension.h>

namespace llmt {
std::vector<at::Tensor> add_rmsnorm_fwd(c10::optional<at::Tensor> a, at::Tensor r, at::Tensor w, double eps,
                                        bool write_s);
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor s, at::Tensor w, at::Tensor rstd,
                                    c10::optional<at::Tensor> ds_in, at::Tensor dw, at::Tensor ticket,
                                    bool write_ds16, bool accumulate);
void swiglu_fwd(at::Tensor g, at::Tensor u, at::Tensor h);
void swiglu_bwd(at::Tensor dh, at::Tensor g, at::Tensor u, at::Tensor dg, at::Tensor du);
void rope_inplace(at::Tensor qkv, at::Tensor cos_t, at::Tensor sin_t, int64_t T, int64_t n_rot_heads, int64_t hd,
                  bool backward);
void embedding_fwd(at::Tensor idx, at::Tensor W, at::Tensor x, c10::optional<at::Tensor> err);
void embedding_bwd(at::Tensor idx, at::Tensor dx, at::Tensor dW);
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p16,
                at::Tensor lr, at::Tensor step, double b1, double b2, double eps, double wd, double grad_scale);
void cast_bf16(at::Tensor x, at::Tensor y);
void ce_fwd_rows(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor loss);
void ce_bwd_rows(at::Tensor logits, at::Tensor targets, at::Tensor lse, c10::optional<at::Tensor> grad_out,
                 double scale);
void gemm(at::Tensor a, at::Tensor b, bool ta, bool tb, int64_t epi, at::Tensor out, bool accumulate,
          c10::optional<at::Tensor> aux, c10::optional<at::Tensor> out2, int64_t split,
          c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t, int64_t T, int64_t hd, int64_t rot_cols,
          c10::optional<at::Tensor> tgt, c10::optional<at::Tensor> lse, c10::optional<at::Tensor> grad_out,
          c10::optional<at::Tensor> part, c10::optional<at::Tensor> tlogit, double alpha, int64_t bn);
int gemm_error_code(bool reset);
void ce_combine(at::Tensor part, at::Tensor tlogit, at::Tensor tgt, at::Tensor lse, at::Tensor loss, int64_t nblk,
                int64_t V);
std::vector<at::Tensor> flash_attn_fwd(at::Tensor qkv, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd,
                                       bool causal, double scale);
at::Tensor flash_attn_bwd(at::Tensor dO, at::Tensor qkv, at::Tensor o, at::Tensor lse, at::Tensor cos_t,
                          at::Tensor sin_t, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd, bool causal,
                          double scale);
int attn_error_code(bool reset);
}  // namespace llmt

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  using namespace pybind11::literals;
  m.doc() = "llmt native sm_100a kernels";
  m.def("add_rmsnorm_fwd", &llmt::add_rmsnorm_fwd, "a"_a, "r"_a, "w"_a, "eps"_a, "write_s"_a);
  m.def("rmsnorm_bwd", &llmt::rmsnorm_bwd, "dy"_a, "s"_a, "w"_a, "rstd"_a, "ds_in"_a, "dw"_a, "ticket"_a,
        "write_ds16"_a, "accumulate"_a);
  m.def("swiglu_fwd", &llmt::swiglu_fwd);
  m.def("swiglu_bwd", &llmt::swiglu_bwd);
  m.def("rope_inplace", &llmt::rope_inplace);
  m.def("embedding_fwd", &llmt::embedding_fwd);
  m.def("embedding_bwd", &llmt::embedding_bwd);
  m.def("adamw_step", &llmt::adamw_step);
  m.def("cast_bf16", &llmt::cast_bf16);
  m.def("ce_fwd_rows", &llmt::ce_fwd_rows);
  m.def("ce_bwd_rows", &llmt::ce_bwd_rows);
  m.def("gemm", &llmt::gemm, "a"_a, "b"_a, "ta"_a, "tb"_a, "epi"_a, "out"_a, "accumulate"_a = false,
        "aux"_a = py::none(), "out2"_a = py::none(), "split"_a = 0, "cos_t"_a = py::none(), "sin_t"_a = py::none(),
        "T"_a = 0, "hd"_a = 0, "rot_cols"_a = 0, "tgt"_a = py::none(), "lse"_a = py::none(),
        "grad_out"_a = py::none(), "part"_a = py::none(), "tlogit"_a = py::none(), "alpha"_a = 1.0, "bn"_a = 0);
  m.def("gemm_error_code", &llmt::gemm_error_code, "reset"_a = false);
  m.def("ce_combine", &llmt::ce_combine);
  m.def("flash_attn_fwd", &llmt::flash_attn_fwd);
  m.def("flash_attn_bwd", &llmt::flash_attn_bwd);
  m.def("attn_error_code", &llmt::attn_error_code, "reset"_a = false);
}

// Python bindings of the dion_b200 CUDA extension (module dion_b200._C).
#include <torch/extension.h>

#include <tuple>

#include "host_utils.h"

namespace bdion {
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C, double alpha,
          double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow, bool sym,
          bool param_mode, double gamma, double delta, int64_t bn_pref, const c10::optional<at::Tensor>& D_ptrs,
          int64_t ldd_ptrs, int64_t out_dtype_ptrs);
void gemm_ex(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C,
             double alpha, double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow,
             bool sym, bool param_mode, double gamma, double delta, int64_t bn_pref,
             const c10::optional<at::Tensor>& D_ptrs, int64_t ldd_ptrs, int64_t out_dtype_ptrs, int64_t nrep,
             int64_t rows_per_ptr, int64_t rot_b, int64_t rot_rows);
void set_gemm_pair_mode(int64_t mode);
int gemm_pair_mode();
std::tuple<int64_t, at::Tensor> symm_create(int64_t bytes);
int64_t symm_open(const at::Tensor& handle);
void symm_close(int64_t peer_ptr);
void symm_free(int64_t ptr);
at::Tensor symm_view(int64_t ptr, int64_t numel, int64_t dtype);
void symm_barrier(const at::Tensor& peer_flags, int64_t my_flags, int64_t rank, int64_t world);
void symm_reduce_slots(const at::Tensor& src, at::Tensor& dst, int64_t nslots);
void symm_push(const at::Tensor& src, const at::Tensor& dsts);
int64_t symm_flag_bytes();
void newton_schulz_ex(at::Tensor& U, const at::Tensor& scale, const std::vector<double>& coeffs, at::Tensor& out,
                      bool clobber_input, const c10::optional<at::Tensor>& out_ptrs, int64_t rows_per_ptr,
                      int64_t rot_rows, int64_t nrep);
void newton_schulz(at::Tensor& U, const at::Tensor& scale, const std::vector<double>& coeffs, at::Tensor& out,
                   bool clobber_input);
void muon_momentum(const std::vector<at::Tensor>& M, const std::vector<at::Tensor>& G,
                   const std::vector<at::Tensor>& U, double mu, bool nesterov, at::Tensor& sumsq, at::Tensor& scale,
                   double eps);
void multi_sumsq(const std::vector<at::Tensor>& X, at::Tensor& sumsq);
void scaled_update(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& U, double decay,
                   const at::Tensor& lrs);
void adamw(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& G, const std::vector<at::Tensor>& M,
           const std::vector<at::Tensor>& V, double lr, double beta1, double beta2, double wd, double eps,
           int64_t step, bool cautious);
void lion(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& G, const std::vector<at::Tensor>& M,
          double lr, double beta1, double beta2, double wd, bool cautious);
void rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps);
void rms_norm_bwd(const at::Tensor& gy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                  at::Tensor& gx, at::Tensor& gw);
void add_rms_norm_fwd(const at::Tensor& x, const at::Tensor& a, const at::Tensor& w, at::Tensor& h, at::Tensor& y,
                      at::Tensor& rstd, double eps);
void rms_norm_bwd_res(const at::Tensor& gy, const at::Tensor& h, const at::Tensor& w, const at::Tensor& rstd,
                      const at::Tensor& gres, at::Tensor& gx, at::Tensor& gw);
void rope_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& tab, at::Tensor& qo, at::Tensor& ko,
              bool inverse);
void swiglu_fwd(const at::Tensor& a, const at::Tensor& b, at::Tensor& o);
void swiglu_bwd(const at::Tensor& g, const at::Tensor& a, const at::Tensor& b, at::Tensor& ga, at::Tensor& gb);
void cross_entropy_fwd_bwd(const at::Tensor& logits, const at::Tensor& labels, at::Tensor& grad, at::Tensor& loss,
                           double scale);
void dion_momentum_add(const std::vector<at::Tensor>& M, const std::vector<at::Tensor>& G, at::Tensor& nz);
void dion_fixup(at::Tensor& P, at::Tensor& R, const at::Tensor& Q0, const at::Tensor& nz);
void col_sumsq(const at::Tensor& R, at::Tensor& out);
void col_normalize(const at::Tensor& R, const at::Tensor& sumsq, double eps, at::Tensor& Q);
void philox_normal(at::Tensor& out, int64_t key, int64_t stream, double scale);
void effective_rank(const at::Tensor& sumsq, const at::Tensor& slots, const at::Tensor& ranks, at::Tensor& out);
void cholesky_lower(at::Tensor& A, at::Tensor& info);
void tri_inv_lower(const at::Tensor& S, at::Tensor& Z, bool upper);
void qr_r(at::Tensor& A, at::Tensor& R);
void qr_r_blocked(at::Tensor& A, at::Tensor& R);
void cholesky_blocked(at::Tensor& A, at::Tensor& info);
void dion2_row_scores(const at::Tensor& ptrs, int64_t rows, int64_t cols, int64_t ld, int64_t dtype,
                      at::Tensor& scores);
void dion2_topk_rows(const at::Tensor& scores, int64_t k, at::Tensor& idx, at::Tensor& pos);
void dion2_gather_decay(const at::Tensor& ptrs, int64_t cols, int64_t ld, int64_t dtype, const at::Tensor& idx,
                        double decay, at::Tensor& sel);
void dion2_update(const at::Tensor& ptrs, int64_t rows, int64_t cols, int64_t ld, int64_t dtype,
                  const at::Tensor& pos, const at::Tensor& U, double keep, double alpha);
}  // namespace bdion

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dion_b200 sm_100a kernels";
  m.def("gemm", &bdion::gemm, "tcgen05 batched bf16 GEMM with fused epilogue", py::arg("A"), py::arg("B"),
        py::arg("D"), py::arg("C") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
        py::arg("scale") = py::none(), py::arg("alpha_pow") = 0, py::arg("beta_pow") = 0, py::arg("sym") = false,
        py::arg("param_mode") = false, py::arg("gamma") = 1.0, py::arg("delta") = 1.0, py::arg("bn") = 0,
        py::arg("D_ptrs") = py::none(), py::arg("ldd_ptrs") = 0, py::arg("out_dtype_ptrs") = 0);
  m.def("gemm_ex", &bdion::gemm_ex, "gemm with replicated / row-split pointer-array outputs", py::arg("A"),
        py::arg("B"), py::arg("D"), py::arg("C"), py::arg("alpha"), py::arg("beta"), py::arg("scale"),
        py::arg("alpha_pow"), py::arg("beta_pow"), py::arg("sym"), py::arg("param_mode"), py::arg("gamma"),
        py::arg("delta"), py::arg("bn"), py::arg("D_ptrs"), py::arg("ldd_ptrs"), py::arg("out_dtype_ptrs"),
        py::arg("nrep"), py::arg("rows_per_ptr"), py::arg("rot_b") = 0, py::arg("rot_rows") = 0);
  m.def("set_gemm_pair_mode", &bdion::set_gemm_pair_mode, "CTA-pair GEMM kernels on (1) / off (0)");
  m.def("gemm_pair_mode", &bdion::gemm_pair_mode);
  m.def("symm_create", &bdion::symm_create);
  m.def("symm_open", &bdion::symm_open);
  m.def("symm_close", &bdion::symm_close);
  m.def("symm_free", &bdion::symm_free);
  m.def("symm_view", &bdion::symm_view);
  m.def("symm_barrier", &bdion::symm_barrier);
  m.def("symm_reduce_slots", &bdion::symm_reduce_slots);
  m.def("symm_push", &bdion::symm_push);
  m.def("symm_flag_bytes", &bdion::symm_flag_bytes);
  m.def("newton_schulz", &bdion::newton_schulz, "batched quintic Newton-Schulz", py::arg("U"), py::arg("scale"),
        py::arg("coeffs"), py::arg("out"), py::arg("clobber_input") = false);
  m.def("newton_schulz_ex", &bdion::newton_schulz_ex, "Newton-Schulz whose last GEMM scatters rows",
        py::arg("U"), py::arg("scale"), py::arg("coeffs"), py::arg("out"), py::arg("clobber_input"),
        py::arg("out_ptrs"), py::arg("rows_per_ptr"), py::arg("rot_rows") = 0, py::arg("nrep") = 1);
  m.def("muon_momentum", &bdion::muon_momentum);
  m.def("multi_sumsq", &bdion::multi_sumsq);
  m.def("scaled_update", &bdion::scaled_update);
  m.def("adamw", &bdion::adamw);
  m.def("lion", &bdion::lion);
  m.def("rms_norm_fwd", &bdion::rms_norm_fwd);
  m.def("rms_norm_bwd", &bdion::rms_norm_bwd);
  m.def("add_rms_norm_fwd", &bdion::add_rms_norm_fwd, "h = x + a, y = rms_norm(h) * w (one pass)");
  m.def("rms_norm_bwd_res", &bdion::rms_norm_bwd_res, "RMSNorm backward plus a residual gradient");
  m.def("rope_fwd", &bdion::rope_fwd);
  m.def("swiglu_fwd", &bdion::swiglu_fwd);
  m.def("swiglu_bwd", &bdion::swiglu_bwd);
  m.def("cross_entropy_fwd_bwd", &bdion::cross_entropy_fwd_bwd);
  m.def("dion_momentum_add", &bdion::dion_momentum_add);
  m.def("dion_fixup", &bdion::dion_fixup);
  m.def("col_sumsq", &bdion::col_sumsq);
  m.def("col_normalize", &bdion::col_normalize);
  m.def("effective_rank", &bdion::effective_rank);
  m.def("philox_normal", &bdion::philox_normal, "counter-based N(0, scale^2) fill (Philox-4x32-10 + Box-Muller)");
  m.def("cholesky_lower", &bdion::cholesky_lower);
  m.def("tri_inv_lower", &bdion::tri_inv_lower);
  m.def("qr_r", &bdion::qr_r);
  m.def("qr_r_blocked", &bdion::qr_r_blocked, "blocked Householder QR (R only), tcgen05 3xTF32 trailing update");
  m.def("cholesky_blocked", &bdion::cholesky_blocked, "blocked Cholesky, tcgen05 3xTF32 trailing SYRK");
  m.def("dion2_row_scores", &bdion::dion2_row_scores, "L1 row norms of a set of matrices (pointer array)");
  m.def("dion2_topk_rows", &bdion::dion2_topk_rows, "per-matrix top-k rows (ascending) and row->slot map");
  m.def("dion2_gather_decay", &bdion::dion2_gather_decay, "gather selected rows (bf16) and decay them in place");
  m.def("dion2_update", &bdion::dion2_update, "row-sparse weight update with weight decay on every row");
  m.def("status_read", &bdion::status_read);
  m.def("status_clear", &bdion::status_clear);
  m.def("set_wait_limit_ns", &bdion::set_wait_limit_ns);
  m.def("wait_limit_ns", &bdion::wait_limit_ns);
  m.def("launch_count", &bdion::launch_count);
}

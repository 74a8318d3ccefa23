// Python bindings of the dion_b200 CUDA extension (module dion_b200._C).
#include <torch/extension.h>

#include "host_utils.h"

namespace bdion {
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C, double alpha,
          double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow, bool sym,
          bool param_mode, double gamma, double delta, int64_t bn_pref);
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
}  // namespace bdion

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dion_b200 sm_100a kernels";
  m.def("gemm", &bdion::gemm, "tcgen05 batched bf16 GEMM with fused epilogue", py::arg("A"), py::arg("B"),
        py::arg("D"), py::arg("C") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
        py::arg("scale") = py::none(), py::arg("alpha_pow") = 0, py::arg("beta_pow") = 0, py::arg("sym") = false,
        py::arg("param_mode") = false, py::arg("gamma") = 1.0, py::arg("delta") = 1.0, py::arg("bn") = 0);
  m.def("newton_schulz", &bdion::newton_schulz, "batched quintic Newton-Schulz", py::arg("U"), py::arg("scale"),
        py::arg("coeffs"), py::arg("out"), py::arg("clobber_input") = false);
  m.def("muon_momentum", &bdion::muon_momentum);
  m.def("multi_sumsq", &bdion::multi_sumsq);
  m.def("scaled_update", &bdion::scaled_update);
  m.def("adamw", &bdion::adamw);
  m.def("lion", &bdion::lion);
  m.def("status_read", &bdion::status_read);
  m.def("status_clear", &bdion::status_clear);
  m.def("set_wait_limit_ns", &bdion::set_wait_limit_ns);
  m.def("wait_limit_ns", &bdion::wait_limit_ns);
}

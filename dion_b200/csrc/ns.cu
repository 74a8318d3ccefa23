// Batched quintic Newton-Schulz orthogonalisation on the tcgen05 GEMM.
//
// For each matrix U_b (m x n) with scale s_b = 1/(||U_b||_F + eps):
//   X_0 = s_b U_b
//   repeat for (a, b, c) in coeffs:
//     A = X X^T          (symmetric: upper tiles only, mirrored)
//     B = b A + c A A    (symmetric)
//     X = a X + B X
// For tall matrices (m > n) the same iteration runs on X^T without a
// transpose copy: A = X^T X, B as above, X = a X + X B (operand layouts are
// picked through the GEMM's K-/MN-major tensor maps).
// The Frobenius scaling of the first iteration is folded into the GEMM
// epilogues (alpha/beta scaled by s_b^k), so U is read unnormalised.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <tuple>
#include <vector>

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

// U: [batch, m, n] bf16 contiguous (not normalised). scale: [batch] fp32.
// out: [batch, m, n] bf16. If clobber_input, U may be used as scratch.
// With out_ptrs the last iteration's GEMM does not write `out`: rows
// [j*rows_per_ptr, (j+1)*rows_per_ptr) of matrix b go to
// out_ptrs[(b*splits + j)*nrep + rep] for rep < nrep (row stride n), e.g.
// straight into the ranks that own those rows, or into every rank.
void newton_schulz_ex(at::Tensor& U, const at::Tensor& scale, const std::vector<double>& coeffs, at::Tensor& out,
                      bool clobber_input, const c10::optional<at::Tensor>& out_ptrs, int64_t rows_per_ptr,
                      int64_t rot_rows, int64_t nrep) {
  TORCH_CHECK(U.dim() == 3 && U.is_contiguous() && U.scalar_type() == at::kBFloat16,
              "dion_b200 newton_schulz: U must be a contiguous [batch, m, n] bf16 tensor");
  TORCH_CHECK(out.sizes() == U.sizes() && out.is_contiguous() && out.scalar_type() == at::kBFloat16,
              "dion_b200 newton_schulz: out must match U");
  TORCH_CHECK(coeffs.size() % 3 == 0 && !coeffs.empty(), "dion_b200 newton_schulz: coeffs must be (a,b,c) triples");
  TORCH_CHECK(out.data_ptr() != U.data_ptr(), "dion_b200 newton_schulz: out must not alias U");
  c10::cuda::CUDAGuard guard(U.device());
  const int64_t bsz = U.size(0), m = U.size(1), n = U.size(2);
  const bool tall = m > n;
  const int64_t s = tall ? n : m;
  const int iters = (int)(coeffs.size() / 3);

  auto opts = U.options();
  at::Tensor A = at::empty({bsz, s, s}, opts);
  at::Tensor Bm = at::empty({bsz, s, s}, opts);
  at::Tensor tmp;
  const bool need_ws = !clobber_input || (iters % 2 == 0);
  tmp = need_ws ? at::empty_like(U) : U;

  auto dst_of = [&](int i) -> at::Tensor& { return ((iters - 1 - i) % 2 == 0) ? out : tmp; };
  at::Tensor src = U;
  const c10::optional<at::Tensor> none;
  for (int i = 0; i < iters; ++i) {
    const double a = coeffs[3 * i], b = coeffs[3 * i + 1], c = coeffs[3 * i + 2];
    const bool first = i == 0;
    const c10::optional<at::Tensor> sc = first ? c10::optional<at::Tensor>(scale) : none;
    at::Tensor& dst = dst_of(i);
    if (!tall) {
      // A = X X^T : A-operand X [m,K=n] K-major; B-operand X^T [K=n, N=m] -> view of X, K-major
      gemm(src, src.transpose(1, 2), A, none, 1.0, 0.0, sc, 2, 0, true, false, 0, 0, 0, none, 0, 0);
      // B = b A + c A A
      gemm(A, A.transpose(1, 2), Bm, A, c, b, none, 0, 0, true, false, 0, 0, 0, none, 0, 0);
      // X' = a X + B X : B-operand X [K=m, N=n] N-major
      if (i == iters - 1 && out_ptrs.has_value())
        gemm_ex(Bm, src, dst, src, 1.0, a, sc, 1, 1, false, false, 0, 0, 0, out_ptrs, n, (int64_t)at::kBFloat16,
                nrep, rows_per_ptr, 0, rot_rows);
      else
        gemm(Bm, src, dst, src, 1.0, a, sc, 1, 1, false, false, 0, 0, 0, none, 0, 0);
    } else {
      // A = X^T X : A-operand X^T [n, K=m] (MN-major view); B-operand X [K=m, N=n] N-major
      gemm(src.transpose(1, 2), src, A, none, 1.0, 0.0, sc, 2, 0, true, false, 0, 0, 0, none, 0, 0);
      gemm(A, A.transpose(1, 2), Bm, A, c, b, none, 0, 0, true, false, 0, 0, 0, none, 0, 0);
      // X' = a X + X B : A-operand X [m, K=n] K-major; B-operand B [K=n, N=n] (symmetric) K-major view
      if (i == iters - 1 && out_ptrs.has_value())
        gemm_ex(src, Bm.transpose(1, 2), dst, src, 1.0, a, sc, 1, 1, false, false, 0, 0, 0, out_ptrs, n,
                (int64_t)at::kBFloat16, nrep, rows_per_ptr, 0, rot_rows);
      else
        gemm(src, Bm.transpose(1, 2), dst, src, 1.0, a, sc, 1, 1, false, false, 0, 0, 0, none, 0, 0);
    }
    src = dst;
  }
}

void newton_schulz(at::Tensor& U, const at::Tensor& scale, const std::vector<double>& coeffs, at::Tensor& out,
                   bool clobber_input) {
  newton_schulz_ex(U, scale, coeffs, out, clobber_input, c10::nullopt, 0, 0, 1);
}

}  // namespace bdion

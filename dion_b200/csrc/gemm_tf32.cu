// fp32-operand (tcgen05 kind::tf32) instantiations of the GEMM kernel, used
// by the Dion power iteration on fp32 momentum / Q / P and by the
// orthogonalisation (sketch, triangular solve, Gram matrix).
#include "gemm_launch.cuh"

namespace bdion {

void gemm_dispatch_tf32(bool a_mn, bool b_mn, int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb,
                        const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param) {
  using bf = __nv_bfloat16;
  if (param) {
    if (out == at::kFloat)
      gemm_launch_major<float, float, bf, true>(a_mn, b_mn, bn, pair, ma, mb, args, s);
    else
      gemm_launch_major<float, bf, bf, true>(a_mn, b_mn, bn, pair, ma, mb, args, s);
  } else {
    TORCH_CHECK(out == at::kFloat, "dion_b200 gemm: tf32 path writes fp32 (store mode)");
    gemm_launch_major<float, float, float, false>(a_mn, b_mn, bn, pair, ma, mb, args, s);
  }
}

}  // namespace bdion

// bf16-operand (tcgen05 kind::f16) instantiations of the GEMM kernel.
#include "gemm_launch.cuh"

namespace bdion {

void gemm_dispatch_bf16(bool a_mn, bool b_mn, int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb,
                        const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param) {
  using bf = __nv_bfloat16;
  if (param) {
    if (out == at::kFloat)
      gemm_launch_major<bf, float, bf, true>(a_mn, b_mn, bn, pair, ma, mb, args, s);
    else
      gemm_launch_major<bf, bf, bf, true>(a_mn, b_mn, bn, pair, ma, mb, args, s);
  } else {
    if (out == at::kFloat)
      gemm_launch_major<bf, float, float, false>(a_mn, b_mn, bn, pair, ma, mb, args, s);
    else
      gemm_launch_major<bf, bf, bf, false>(a_mn, b_mn, bn, pair, ma, mb, args, s);
  }
}

}  // namespace bdion

// bf16-operand (tcgen05 kind::f16) instantiations of the single-CTA GEMM kernel.
#include "gemm_launch.cuh"

namespace bdion {

void gemm_dispatch_bf16_single(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args,
            cudaStream_t s, at::ScalarType out, bool param) {
  gemm_dispatch_bf16_impl<false>(a_mn, b_mn, bn, ma, mb, args, s, out, param);
}

}  // namespace bdion

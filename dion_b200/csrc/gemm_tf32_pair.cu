// fp32-operand (tcgen05 kind::tf32) instantiations of the CTA-pair GEMM kernel.
#include "gemm_launch.cuh"

namespace bdion {

void gemm_dispatch_tf32_pair(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args,
            cudaStream_t s, at::ScalarType out, bool param) {
  gemm_dispatch_tf32_impl<true>(a_mn, b_mn, bn, ma, mb, args, s, out, param);
}

}  // namespace bdion

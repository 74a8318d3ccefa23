// Templated launch helpers of the tcgen05 GEMM, shared by the translation
// units that instantiate the bf16 (kind::f16) and fp32 (kind::tf32) kernels.
#pragma once
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>

#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "host_utils.h"

namespace bdion {

int gemm_sm_count();

template <typename TIn, int BN, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void gemm_launch_typed(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<TIn, BN, A_MN, B_MN, OutT, CT, PARAM>;
  constexpr int smem = GemmCfg<BN>::kSmemBytes;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  const int grid = std::min(args.total_tiles, gemm_sm_count());
  kern<<<grid, 192, smem, stream>>>(ma, mb, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// CTA-pair kernel: clusters of 2, one pair per two SMs, persistent over tiles.
template <typename TIn, int BN, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void gemm_launch_typed2(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, cudaStream_t stream) {
  auto kern = gemm_tc2_kernel<TIn, BN, A_MN, B_MN, OutT, CT, PARAM>;
  constexpr int smem = GemmCfg2<BN>::kSmemBytes;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  const int pairs = std::max(1, std::min(args.total_tiles, gemm_sm_count() / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ma, mb, args));
  note_launch();
}

template <typename TIn, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void gemm_launch_bn(int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args,
                    cudaStream_t s) {
  if (pair) {
    if (bn == 256)
      gemm_launch_typed2<TIn, 256, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
    else
      gemm_launch_typed2<TIn, 128, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
    return;
  }
  if (bn == 256)
    gemm_launch_typed<TIn, 256, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
  else
    gemm_launch_typed<TIn, 128, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
}

template <typename TIn, typename OutT, typename CT, bool PARAM>
void gemm_launch_major(bool a_mn, bool b_mn, int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb,
                       const GemmArgs& args, cudaStream_t s) {
  if (!a_mn && !b_mn)
    gemm_launch_bn<TIn, false, false, OutT, CT, PARAM>(bn, pair, ma, mb, args, s);
  else if (!a_mn && b_mn)
    gemm_launch_bn<TIn, false, true, OutT, CT, PARAM>(bn, pair, ma, mb, args, s);
  else if (a_mn && !b_mn)
    gemm_launch_bn<TIn, true, false, OutT, CT, PARAM>(bn, pair, ma, mb, args, s);
  else
    gemm_launch_bn<TIn, true, true, OutT, CT, PARAM>(bn, pair, ma, mb, args, s);
}

// Entry points implemented in gemm_bf16.cu / gemm_tf32.cu.
// mode: 0 = store (OutT = out dtype, CT = OutT), 1 = param update
void gemm_dispatch_bf16(bool a_mn, bool b_mn, int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb,
                        const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param);
void gemm_dispatch_tf32(bool a_mn, bool b_mn, int bn, bool pair, const CUtensorMap& ma, const CUtensorMap& mb,
                        const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param);

}  // namespace bdion

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

template <bool PAIR, typename TIn, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void gemm_launch_bn(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, cudaStream_t s) {
  if constexpr (PAIR) {
    if (bn == 256)
      gemm_launch_typed2<TIn, 256, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
    else
      gemm_launch_typed2<TIn, 128, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
  } else {
    if (bn == 256)
      gemm_launch_typed<TIn, 256, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
    else
      gemm_launch_typed<TIn, 128, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
  }
}

template <bool PAIR, typename TIn, typename OutT, typename CT, bool PARAM>
void gemm_launch_major(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                       const GemmArgs& args, cudaStream_t s) {
  if (!a_mn && !b_mn)
    gemm_launch_bn<PAIR, TIn, false, false, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else if (!a_mn && b_mn)
    gemm_launch_bn<PAIR, TIn, false, true, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else if (a_mn && !b_mn)
    gemm_launch_bn<PAIR, TIn, true, false, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else
    gemm_launch_bn<PAIR, TIn, true, true, OutT, CT, PARAM>(bn, ma, mb, args, s);
}

// Per-input-type instantiations, one translation unit per (type, kernel
// family) so the build compiles them in parallel.
template <bool PAIR>
void gemm_dispatch_bf16_impl(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                             const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param) {
  using bf = __nv_bfloat16;
  if (param) {
    if (out == at::kFloat)
      gemm_launch_major<PAIR, bf, float, bf, true>(a_mn, b_mn, bn, ma, mb, args, s);
    else
      gemm_launch_major<PAIR, bf, bf, bf, true>(a_mn, b_mn, bn, ma, mb, args, s);
  } else {
    if (out == at::kFloat)
      gemm_launch_major<PAIR, bf, float, float, false>(a_mn, b_mn, bn, ma, mb, args, s);
    else
      gemm_launch_major<PAIR, bf, bf, bf, false>(a_mn, b_mn, bn, ma, mb, args, s);
  }
}

template <bool PAIR>
void gemm_dispatch_tf32_impl(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                             const GemmArgs& args, cudaStream_t s, at::ScalarType out, bool param) {
  using bf = __nv_bfloat16;
  if (param) {
    if (out == at::kFloat)
      gemm_launch_major<PAIR, float, float, bf, true>(a_mn, b_mn, bn, ma, mb, args, s);
    else
      gemm_launch_major<PAIR, float, bf, bf, true>(a_mn, b_mn, bn, ma, mb, args, s);
  } else {
    TORCH_CHECK(out == at::kFloat, "dion_b200 gemm: tf32 path writes fp32 (store mode)");
    gemm_launch_major<PAIR, float, float, float, false>(a_mn, b_mn, bn, ma, mb, args, s);
  }
}

#define BDION_GEMM_DISPATCH_DECL(name)                                                                   \
  void name(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, \
            cudaStream_t s, at::ScalarType out, bool param);
BDION_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_single)
BDION_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_pair)
BDION_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_single)
BDION_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_pair)
#undef BDION_GEMM_DISPATCH_DECL

}  // namespace bdion

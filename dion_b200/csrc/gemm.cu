// Host side of the tcgen05 GEMM: tensor-map construction, tile-count
// bookkeeping, kernel selection and launch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "gemm_tc.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "dion_b200: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 tensor map over storage [batch][rows][cols] (cols contiguous),
// box = {64 cols, box_rows rows, 1}, 128-byte swizzle, zero fill out of bounds.
CUtensorMap make_map_bf16(const void* base, int64_t cols, int64_t rows, int64_t batch, int64_t ld, int64_t bstride,
                          int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  if (batch <= 1) bstride = ld * rows;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(bstride * 2)};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "dion_b200 gemm: operand base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0 && (bstride * 2) % 16 == 0,
              "dion_b200 gemm: operand row/batch strides must be multiples of 16 bytes (ld % 8 == 0)");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "dion_b200 gemm: cuTensorMapEncodeTiled failed with ", (int)r);
  return m;
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

template <int BN, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void launch_typed(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, OutT, CT, PARAM>;
  constexpr int smem = GemmCfg<BN>::kSmemBytes;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  const int grid = std::min(args.total_tiles, sm_count());
  kern<<<grid, 192, smem, stream>>>(ma, mb, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
void launch_bn(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args, cudaStream_t s) {
  if (bn == 256)
    launch_typed<256, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
  else
    launch_typed<128, A_MN, B_MN, OutT, CT, PARAM>(ma, mb, args, s);
}

template <typename OutT, typename CT, bool PARAM>
void launch_major(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args,
                  cudaStream_t s) {
  if (!a_mn && !b_mn)
    launch_bn<false, false, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else if (!a_mn && b_mn)
    launch_bn<false, true, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else if (a_mn && !b_mn)
    launch_bn<true, false, OutT, CT, PARAM>(bn, ma, mb, args, s);
  else
    launch_bn<true, true, OutT, CT, PARAM>(bn, ma, mb, args, s);
}

}  // namespace

// A: [batch, M, K] bf16 view, B: [batch, K, N] bf16 view (any layout with one
// unit stride in the last two dims); D: [batch, M, N] row-major output.
// param_mode: D = gamma*D + delta*(alpha*A@B + beta*C) in place.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C, double alpha,
          double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow, bool sym,
          bool param_mode, double gamma, double delta, int64_t bn_pref) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda(), "dion_b200 gemm: CUDA tensors expected");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && D.dim() == 3, "dion_b200 gemm: 3-D [batch, rows, cols] views expected");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "dion_b200 gemm: bf16 operands expected");
  const int64_t batch = A.size(0), M = A.size(1), K = A.size(2), N = B.size(2);
  TORCH_CHECK(B.size(0) == batch && B.size(1) == K, "dion_b200 gemm: shape mismatch");
  TORCH_CHECK(D.size(0) == batch && D.size(1) == M && D.size(2) == N && D.stride(2) == 1,
              "dion_b200 gemm: D must be [batch, M, N] with unit column stride");
  TORCH_CHECK(K > 0 && M > 0 && N > 0, "dion_b200 gemm: empty problem");
  c10::cuda::CUDAGuard guard(A.device());

  // Operand majors from strides.
  const bool a_mn = A.stride(2) != 1;  // A stored [K][M]
  const bool b_mn = B.stride(2) == 1;  // B stored [K][N] (N contiguous)
  TORCH_CHECK(a_mn ? A.stride(1) == 1 : A.stride(2) == 1, "dion_b200 gemm: A needs a unit stride");
  TORCH_CHECK(b_mn ? B.stride(2) == 1 : B.stride(1) == 1, "dion_b200 gemm: B needs a unit stride");
  if (sym) TORCH_CHECK(M == N && !param_mode, "dion_b200 gemm: symmetric mode needs a square output");

  int bn = (bn_pref == 128 || bn_pref == 256) ? (int)bn_pref : (N > 128 ? 256 : 128);
  CUtensorMap ma = a_mn ? make_map_bf16(A.data_ptr(), M, K, batch, A.stride(2), A.stride(0), 64)
                        : make_map_bf16(A.data_ptr(), K, M, batch, A.stride(1), A.stride(0), kBM);
  CUtensorMap mb = b_mn ? make_map_bf16(B.data_ptr(), N, K, batch, B.stride(1), B.stride(0), 64)
                        : make_map_bf16(B.data_ptr(), K, N, batch, B.stride(2), B.stride(0), bn);

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.batch = (int)batch;
  args.D = D.data_ptr();
  args.ldd = D.stride(1);
  args.strideD = D.stride(0);
  args.C = nullptr;
  if (C.has_value() && C->defined()) {
    TORCH_CHECK(C->dim() == 3 && C->size(0) == batch && C->size(1) == M && C->size(2) == N && C->stride(2) == 1,
                "dion_b200 gemm: C must be [batch, M, N] with unit column stride");
    args.C = C->data_ptr();
    args.ldc = C->stride(1);
    args.strideC = C->stride(0);
  }
  args.alpha = (float)alpha;
  args.beta = (float)beta;
  args.scale = nullptr;
  if (scale.has_value() && scale->defined()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() >= batch, "dion_b200 gemm: bad scale vector");
    args.scale = scale->data_ptr<float>();
  }
  args.alpha_pow = (int)alpha_pow;
  args.beta_pow = (int)beta_pow;
  args.gamma = (float)gamma;
  args.delta = (float)delta;
  args.sym = sym ? 1 : 0;
  args.tiles_m = (int)((M + kBM - 1) / kBM);
  args.tiles_n = (int)((N + bn - 1) / bn);
  if (sym) {
    int cnt = 0;
    for (int tm = 0; tm < args.tiles_m; ++tm) cnt += args.tiles_n - (tm * kBM) / bn;
    args.tiles_per_batch = cnt;
  } else {
    args.tiles_per_batch = args.tiles_m * args.tiles_n;
  }
  args.total_tiles = args.tiles_per_batch * (int)batch;
  args.status = status_device_ptr();
  args.limit_ns = wait_limit_ns();

  // vector epilogue accesses need 16-byte aligned rows
  auto aligned16 = [](const void* p, int64_t ld, int64_t bs, int esz) {
    return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (ld * esz) % 16 == 0 && (bs * esz) % 16 == 0;
  };
  const int dsz = D.element_size();
  TORCH_CHECK(aligned16(args.D, args.ldd, batch > 1 ? args.strideD : 0, dsz), "dion_b200 gemm: D rows must be 16B aligned");
  if (args.C) TORCH_CHECK(aligned16(args.C, args.ldc, batch > 1 ? args.strideC : 0, C->element_size()),
                          "dion_b200 gemm: C rows must be 16B aligned");

  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const auto dt = D.scalar_type();
  const bool c_bf16 = !args.C || C->scalar_type() == at::kBFloat16;
  if (param_mode) {
    TORCH_CHECK(c_bf16, "dion_b200 gemm: param mode expects a bf16 C");
    if (dt == at::kFloat)
      launch_major<float, __nv_bfloat16, true>(a_mn, b_mn, bn, ma, mb, args, s);
    else if (dt == at::kBFloat16)
      launch_major<__nv_bfloat16, __nv_bfloat16, true>(a_mn, b_mn, bn, ma, mb, args, s);
    else
      TORCH_CHECK(false, "dion_b200 gemm: param dtype must be fp32 or bf16");
  } else {
    if (dt == at::kBFloat16) {
      TORCH_CHECK(c_bf16, "dion_b200 gemm: C must match D dtype");
      launch_major<__nv_bfloat16, __nv_bfloat16, false>(a_mn, b_mn, bn, ma, mb, args, s);
    } else if (dt == at::kFloat) {
      TORCH_CHECK(!args.C || C->scalar_type() == at::kFloat, "dion_b200 gemm: C must match D dtype");
      launch_major<float, float, false>(a_mn, b_mn, bn, ma, mb, args, s);
    } else {
      TORCH_CHECK(false, "dion_b200 gemm: output dtype must be bf16 or fp32");
    }
  }
}

}  // namespace bdion

// Host side of the tcgen05 GEMM: tensor-map construction, tile-count
// bookkeeping, kernel selection and launch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <mutex>

#include "gemm_launch.cuh"

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

// 3-D tensor map over storage [batch][rows][cols] (cols contiguous), box =
// {one 128-byte row of elements, box_rows, 1}, 128-byte swizzle, zero fill
// out of bounds.
CUtensorMap make_map(const void* base, bool fp32, int64_t cols, int64_t rows, int64_t batch, int64_t ld,
                     int64_t bstride, int box_rows, bool mn_major) {
  CUtensorMap m;
  const int esz = fp32 ? 4 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  if (batch <= 1) bstride = ld * rows;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * esz), (cuuint64_t)(bstride * esz)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "dion_b200 gemm: operand base must be 16-byte aligned");
  TORCH_CHECK((ld * esz) % 16 == 0 && (bstride * esz) % 16 == 0,
              "dion_b200 gemm: operand row/batch strides must be multiples of 16 bytes");
  CUresult r = encode_fn()(&m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           (fp32 && mn_major) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "dion_b200 gemm: cuTensorMapEncodeTiled failed with ", (int)r);
  return m;
}

}  // namespace

// CTA-pair (cta_group::2) kernels for problems with at least two 128-row
// tiles: 0 = off, 1 = on. Initial value from DION_B200_GEMM_PAIR (default on; "0" selects the single-CTA kernels).
static int g_pair_mode = -1;
int gemm_pair_mode() {
  if (g_pair_mode < 0) {
    const char* e = std::getenv("DION_B200_GEMM_PAIR");
    g_pair_mode = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pair_mode;
}
void set_gemm_pair_mode(int64_t mode) { g_pair_mode = mode ? 1 : 0; }

int gemm_sm_count() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

// A: [batch, M, K] view, B: [batch, K, N] view (any layout with one unit
// stride in the last two dims), both bf16 (tensor-core bf16) or both fp32
// (tensor-core tf32). D: [batch, M, N] row-major output, or, when D_ptrs is
// given (int64 device tensor of batch addresses), per-batch outputs with row
// stride ldd_ptrs.
// param_mode: D = gamma*D + delta*(alpha*A@B + beta*C) in place.
// nrep / rows_per_ptr: see the pointer-array note in gemm_tc.cuh (D_ptrs
// then holds batch * ceil(M / rows_per_ptr) * nrep addresses).
void gemm_ex(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C,
             double alpha, double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow,
             bool sym, bool param_mode, double gamma, double delta, int64_t bn_pref,
             const c10::optional<at::Tensor>& D_ptrs, int64_t ldd_ptrs, int64_t out_dtype_ptrs, int64_t nrep,
             int64_t rows_per_ptr, int64_t rot_b, int64_t rot_rows) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "dion_b200 gemm: CUDA tensors expected");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3, "dion_b200 gemm: 3-D [batch, rows, cols] views expected");
  const bool fp32_in = A.scalar_type() == at::kFloat;
  TORCH_CHECK((A.scalar_type() == at::kBFloat16 || fp32_in) && B.scalar_type() == A.scalar_type(),
              "dion_b200 gemm: operands must both be bf16 or both fp32");
  const int64_t batch = A.size(0), M = A.size(1), K = A.size(2), N = B.size(2);
  TORCH_CHECK(B.size(0) == batch && B.size(1) == K, "dion_b200 gemm: shape mismatch");
  TORCH_CHECK(K > 0 && M > 0 && N > 0, "dion_b200 gemm: empty problem");
  if (batch == 0) return;  // an empty batch (a rank that holds no matrix of a set)
  const bool use_ptrs = D_ptrs.has_value() && D_ptrs->defined();
  if (!use_ptrs) {
    TORCH_CHECK(D.is_cuda() && D.dim() == 3 && D.size(0) == batch && D.size(1) == M && D.size(2) == N &&
                    D.stride(2) == 1,
                "dion_b200 gemm: D must be [batch, M, N] with unit column stride");
  }
  TORCH_CHECK(nrep >= 1 && rows_per_ptr >= 0, "dion_b200 gemm: bad nrep / rows_per_ptr");
  const int64_t splits = (use_ptrs && rows_per_ptr > 0) ? (M + rows_per_ptr - 1) / rows_per_ptr : 1;
  if (use_ptrs) {
    TORCH_CHECK(D_ptrs->scalar_type() == at::kLong && D_ptrs->numel() >= batch * splits * nrep && D_ptrs->is_cuda(),
                "dion_b200 gemm: D_ptrs must be an int64 CUDA tensor of batch*splits*nrep addresses");
    TORCH_CHECK(!param_mode || nrep == 1, "dion_b200 gemm: param mode writes one destination");
  } else {
    TORCH_CHECK(nrep == 1 && rows_per_ptr == 0, "dion_b200 gemm: nrep / rows_per_ptr need D_ptrs");
  }
  c10::cuda::CUDAGuard guard(A.device());

  const bool a_mn = A.stride(2) != 1;  // A stored [K][M]
  const bool b_mn = B.stride(2) == 1;  // B stored [K][N] (N contiguous)
  TORCH_CHECK(a_mn ? A.stride(1) == 1 : A.stride(2) == 1, "dion_b200 gemm: A needs a unit stride");
  TORCH_CHECK(b_mn ? B.stride(2) == 1 : B.stride(1) == 1, "dion_b200 gemm: B needs a unit stride");
  if (sym) TORCH_CHECK(M == N && !param_mode && !use_ptrs, "dion_b200 gemm: symmetric mode needs a square output");

  const int row_elems = fp32_in ? 32 : 64;  // elements per 128-byte swizzle row
  int bn = (bn_pref == 128 || bn_pref == 256) ? (int)bn_pref : (N > 128 ? 256 : 128);
  // CTA pairs: a 256 x bn tile per pair of SMs, each CTA loading bn/2 columns of B
  const bool pair = gemm_pair_mode() && M > kBM;
  const int bm = pair ? kBM2 : kBM;
  CUtensorMap ma = a_mn ? make_map(A.data_ptr(), fp32_in, M, K, batch, A.stride(2), A.stride(0), row_elems, true)
                        : make_map(A.data_ptr(), fp32_in, K, M, batch, A.stride(1), A.stride(0), kBM, false);
  CUtensorMap mb = b_mn ? make_map(B.data_ptr(), fp32_in, N, K, batch, B.stride(1), B.stride(0), row_elems, true)
                        : make_map(B.data_ptr(), fp32_in, K, N, batch, B.stride(2), B.stride(0), pair ? bn / 2 : bn,
                                   false);

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.batch = (int)batch;
  at::ScalarType out_t;
  if (use_ptrs) {
    args.D = nullptr;
    args.D_ptrs = reinterpret_cast<void* const*>(D_ptrs->data_ptr<int64_t>());
    args.ldd = ldd_ptrs;
    args.strideD = 0;
    out_t = static_cast<at::ScalarType>(out_dtype_ptrs);
  } else {
    args.D = D.data_ptr();
    args.D_ptrs = nullptr;
    args.ldd = D.stride(1);
    args.strideD = D.stride(0);
    out_t = D.scalar_type();
  }
  TORCH_CHECK(rot_b >= 0 && rot_rows >= 0, "dion_b200 gemm: rotations must be non-negative");
  args.rot_b = (int)(batch > 0 ? rot_b % batch : 0);
  args.rot_rows = (int)rot_rows;
  args.nrep = (int)nrep;
  args.rows_per_ptr = use_ptrs ? (int)rows_per_ptr : 0;
  args.splits = (int)splits;
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
  args.tiles_m = (int)((M + bm - 1) / bm);
  args.tiles_n = (int)((N + bn - 1) / bn);
  if (sym) {
    int cnt = 0;
    for (int tm = 0; tm < args.tiles_m; ++tm) cnt += args.tiles_n - (tm * bm) / bn;
    args.tiles_per_batch = cnt;
  } else {
    args.tiles_per_batch = args.tiles_m * args.tiles_n;
  }
  args.total_tiles = args.tiles_per_batch * (int)batch;
  args.status = status_device_ptr();
  args.limit_ns = wait_limit_ns();

  auto aligned16 = [](const void* p, int64_t ld, int64_t bs, int esz) {
    return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (ld * esz) % 16 == 0 && (bs * esz) % 16 == 0;
  };
  const int dsz = (out_t == at::kFloat) ? 4 : 2;
  if (!use_ptrs) {
    TORCH_CHECK(aligned16(args.D, args.ldd, batch > 1 ? args.strideD : 0, dsz), "dion_b200 gemm: D rows must be 16B aligned");
  } else {
    TORCH_CHECK((args.ldd * dsz) % 16 == 0, "dion_b200 gemm: D rows must be 16B aligned");
  }
  if (args.C) {
    TORCH_CHECK(aligned16(args.C, args.ldc, batch > 1 ? args.strideC : 0, C->element_size()),
                "dion_b200 gemm: C rows must be 16B aligned");
  }
  if (args.C && !param_mode) {
    TORCH_CHECK(C->scalar_type() == out_t, "dion_b200 gemm: C must match D dtype");
  }
  if (args.C && param_mode) {
    TORCH_CHECK(C->scalar_type() == at::kBFloat16, "dion_b200 gemm: param mode expects a bf16 C");
  }
  TORCH_CHECK(out_t == at::kFloat || out_t == at::kBFloat16, "dion_b200 gemm: output dtype must be bf16 or fp32");

  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (fp32_in) {
    if (pair)
      gemm_dispatch_tf32_pair(a_mn, b_mn, bn, ma, mb, args, s, out_t, param_mode);
    else
      gemm_dispatch_tf32_single(a_mn, b_mn, bn, ma, mb, args, s, out_t, param_mode);
  } else {
    if (pair)
      gemm_dispatch_bf16_pair(a_mn, b_mn, bn, ma, mb, args, s, out_t, param_mode);
    else
      gemm_dispatch_bf16_single(a_mn, b_mn, bn, ma, mb, args, s, out_t, param_mode);
  }
}

void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C, double alpha,
          double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow, bool sym,
          bool param_mode, double gamma, double delta, int64_t bn_pref, const c10::optional<at::Tensor>& D_ptrs,
          int64_t ldd_ptrs, int64_t out_dtype_ptrs) {
  gemm_ex(A, B, D, C, alpha, beta, scale, alpha_pow, beta_pow, sym, param_mode, gamma, delta, bn_pref, D_ptrs,
          ldd_ptrs, out_dtype_ptrs, 1, 0, 0, 0);
}

}  // namespace bdion

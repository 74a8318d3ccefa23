// Dion2 row selection and sparse update (batched over a set of equally
// shaped matrices; the matrices are separate tensors reached through device
// pointer arrays, so no stacking copy is made):
//
//   dion2_row_scores  : score[b][i] = sum_j |M_b[i][j]|          (L1 row norms)
//   dion2_topk_rows   : the k rows of largest score per matrix, ascending
//                       row order, plus pos[b][i] = slot of row i or -1
//                       (radix select on the float bits, ties to the lowest
//                       rows, two block scans; one CTA per matrix)
//   dion2_gather_decay: sel[b][s] = bf16(M_b[idx[b][s]]) and, in the same
//                       pass, M_b[idx[b][s]] *= ef_decay (selective decay)
//   dion2_update      : X_b[i] = (1 - lr*wd) X_b[i] - adj * U_b[pos[b][i]]
//                       for selected rows, (1 - lr*wd) X_b[i] otherwise
//
// Behaviour (select an alpha-fraction of momentum rows by L1 norm,
// orthogonalise the selected block, decay only the selected rows, apply a
// row-sparse update with weight decay on every row) follows the Dion2
// description the reference uses (paper/main.tex:70; ctor kwargs at
// ada_dion/integration/hybrid_optimizer.py:219-227).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

constexpr int kSelThreads = 1024;

template <typename T>
__global__ void __launch_bounds__(256) row_scores_kernel(const int64_t* __restrict__ ptrs, int rows, int cols,
                                                         int64_t ld, float* __restrict__ scores) {
  const int b = blockIdx.y;
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const T* M = reinterpret_cast<const T*>(ptrs[b]) + (int64_t)row * ld;
  float s = 0.f;
  for (int j = lane; j < cols; j += 32) s += fabsf(to_f<T>(M[j]));
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) scores[(int64_t)b * rows + row] = s;
}

// Block-wide exclusive scan of one int per thread (kSelThreads threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_sums[lane] = t;  // inclusive prefix over warps
  }
  __syncthreads();
  total = warp_sums[31];
  return x - v + (w > 0 ? warp_sums[w - 1] : 0);
}

// One CTA per matrix. Scores are non-negative (or NaN, which sorts above
// every finite score), so their uint32 bit patterns order like the values.
__global__ void __launch_bounds__(kSelThreads) topk_rows_kernel(const float* __restrict__ scores, int rows, int k,
                                                                int64_t* __restrict__ idx, int* __restrict__ pos) {
  extern __shared__ uint32_t sbits[];  // rows
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int b = blockIdx.x;
  const float* sc = scores + (int64_t)b * rows;
  for (int i = threadIdx.x; i < rows; i += kSelThreads) sbits[i] = __float_as_uint(sc[i]) & 0x7fffffffu;
  if (threadIdx.x == 0) {
    s_prefix = 0u;
    s_remaining = k;  // how many of the k still lie among the candidates
  }
  __syncthreads();
  // radix select, most significant byte first: after the 4 passes, s_prefix
  // is the k-th largest bit pattern and s_remaining the number of rows equal
  // to it that belong to the top k
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t pmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    const uint32_t prefix = s_prefix;
    for (int i = threadIdx.x; i < rows; i += kSelThreads) {
      const uint32_t v = sbits[i];
      if ((v & pmask) == prefix) atomicAdd(&hist[(v >> shift) & 0xffu], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int rem = s_remaining, d = 255;
      for (; d > 0; --d) {  // largest digit first
        if (hist[d] >= rem) break;
        rem -= hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_remaining = rem;
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const int need_eq = s_remaining;
  // contiguous strip of rows per thread, so the scans give ascending row order
  const int per = (rows + kSelThreads - 1) / kSelThreads;
  const int lo = threadIdx.x * per, hi = min(rows, lo + per);
  int n_eq = 0;
  for (int i = lo; i < hi; ++i) n_eq += sbits[i] == thr;
  int tot;
  int eq_before = block_exclusive_scan(n_eq, warp_sums, tot);
  int n_sel = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t v = sbits[i];
    if (v > thr) {
      ++n_sel;
    } else if (v == thr) {
      if (eq_before < need_eq) ++n_sel;
      ++eq_before;
    }
  }
  int sel_before = block_exclusive_scan(n_sel, warp_sums, tot);
  eq_before = block_exclusive_scan(n_eq, warp_sums, tot);  // restart the equal-rank count
  int* pb = pos + (int64_t)b * rows;
  int64_t* ib = idx + (int64_t)b * k;
  for (int i = lo; i < hi; ++i) {
    const uint32_t v = sbits[i];
    bool take = false;
    if (v > thr) {
      take = true;
    } else if (v == thr) {
      take = eq_before < need_eq;
      ++eq_before;
    }
    if (take) {
      ib[sel_before] = i;
      pb[i] = sel_before++;
    } else {
      pb[i] = -1;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) gather_decay_kernel(const int64_t* __restrict__ ptrs, int cols, int64_t ld,
                                                           const int64_t* __restrict__ idx, int k, float decay,
                                                           __nv_bfloat16* __restrict__ sel) {
  const int b = blockIdx.y;
  const int s = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (s >= k) return;
  T* row = reinterpret_cast<T*>(ptrs[b]) + idx[(int64_t)b * k + s] * ld;
  __nv_bfloat16* out = sel + ((int64_t)b * k + s) * cols;
  for (int j = lane; j < cols; j += 32) {
    const float v = to_f<T>(row[j]);
    out[j] = __float2bfloat16_rn(v);
    row[j] = from_f<T>(v * decay);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) sparse_update_kernel(const int64_t* __restrict__ ptrs, int rows, int cols,
                                                            int64_t ld, const int* __restrict__ pos,
                                                            const __nv_bfloat16* __restrict__ U, int k, float keep,
                                                            float alpha) {
  const int b = blockIdx.y;
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  T* x = reinterpret_cast<T*>(ptrs[b]) + (int64_t)row * ld;
  const int p = pos[(int64_t)b * rows + row];
  if (p < 0) {
    if (keep != 1.f)
      for (int j = lane; j < cols; j += 32) x[j] = from_f<T>(keep * to_f<T>(x[j]));
    return;
  }
  const __nv_bfloat16* u = U + ((int64_t)b * k + p) * cols;
  for (int j = lane; j < cols; j += 32) x[j] = from_f<T>(keep * to_f<T>(x[j]) - alpha * __bfloat162float(u[j]));
}

#define BDION_D2_DISPATCH(dt, NAME, ...)                          \
  if (dt == at::kFloat) {                                         \
    using NAME = float;                                           \
    __VA_ARGS__                                                   \
  } else if (dt == at::kBFloat16) {                               \
    using NAME = __nv_bfloat16;                                   \
    __VA_ARGS__                                                   \
  } else {                                                        \
    TORCH_CHECK(false, "dion_b200 dion2: fp32 or bf16 matrices"); \
  }

void check_ptrs(const at::Tensor& ptrs) {
  TORCH_CHECK(ptrs.is_cuda() && ptrs.scalar_type() == at::kLong && ptrs.dim() == 1,
              "dion_b200 dion2: pointer array must be a 1-D int64 CUDA tensor");
}

}  // namespace

// ptrs: [n] addresses of row-major (rows x cols, row stride ld) matrices of dtype `dtype`.
void dion2_row_scores(const at::Tensor& ptrs, int64_t rows, int64_t cols, int64_t ld, int64_t dtype,
                      at::Tensor& scores) {
  check_ptrs(ptrs);
  const int n = (int)ptrs.numel();
  TORCH_CHECK(scores.is_cuda() && scores.scalar_type() == at::kFloat && scores.is_contiguous() &&
                  scores.numel() == n * rows,
              "dion_b200 dion2_row_scores: scores must be a contiguous fp32 [n, rows] tensor");
  c10::cuda::CUDAGuard guard(ptrs.device());
  const dim3 grid((unsigned)((rows + 7) / 8), (unsigned)n);
  auto st = at::cuda::getCurrentCUDAStream();
  const auto dt = static_cast<at::ScalarType>(dtype);
  BDION_D2_DISPATCH(dt, T, {
    row_scores_kernel<T><<<grid, 256, 0, st>>>(ptrs.data_ptr<int64_t>(), (int)rows, (int)cols, ld,
                                              scores.data_ptr<float>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// scores: fp32 [n, rows] (non-negative); idx: int64 [n, k] (ascending rows); pos: int32 [n, rows].
void dion2_topk_rows(const at::Tensor& scores, int64_t k, at::Tensor& idx, at::Tensor& pos) {
  TORCH_CHECK(scores.is_cuda() && scores.dim() == 2 && scores.is_contiguous() && scores.scalar_type() == at::kFloat,
              "dion_b200 dion2_topk_rows: contiguous fp32 [n, rows] scores");
  const int n = (int)scores.size(0), rows = (int)scores.size(1);
  TORCH_CHECK(k >= 1 && k <= rows, "dion_b200 dion2_topk_rows: need 1 <= k <= rows");
  TORCH_CHECK(idx.is_contiguous() && idx.scalar_type() == at::kLong && idx.numel() == (int64_t)n * k,
              "dion_b200 dion2_topk_rows: idx must be a contiguous int64 [n, k] tensor");
  TORCH_CHECK(pos.is_contiguous() && pos.scalar_type() == at::kInt && pos.numel() == (int64_t)n * rows,
              "dion_b200 dion2_topk_rows: pos must be a contiguous int32 [n, rows] tensor");
  const size_t smem = (size_t)rows * sizeof(uint32_t);
  TORCH_CHECK(smem <= 200 * 1024, "dion_b200 dion2_topk_rows: at most 51200 rows per matrix");
  c10::cuda::CUDAGuard guard(scores.device());
  C10_CUDA_CHECK(cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  topk_rows_kernel<<<n, kSelThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      scores.data_ptr<float>(), rows, (int)k, idx.data_ptr<int64_t>(), pos.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// sel: bf16 [n, k, cols] contiguous; matrices' selected rows are multiplied by `decay` in place.
void dion2_gather_decay(const at::Tensor& ptrs, int64_t cols, int64_t ld, int64_t dtype, const at::Tensor& idx,
                        double decay, at::Tensor& sel) {
  check_ptrs(ptrs);
  const int n = (int)ptrs.numel();
  TORCH_CHECK(idx.is_cuda() && idx.dim() == 2 && idx.size(0) == n && idx.is_contiguous() &&
                  idx.scalar_type() == at::kLong,
              "dion_b200 dion2_gather_decay: idx must be a contiguous int64 [n, k] tensor");
  const int k = (int)idx.size(1);
  TORCH_CHECK(sel.is_contiguous() && sel.scalar_type() == at::kBFloat16 && sel.numel() == (int64_t)n * k * cols,
              "dion_b200 dion2_gather_decay: sel must be a contiguous bf16 [n, k, cols] tensor");
  c10::cuda::CUDAGuard guard(ptrs.device());
  const dim3 grid((unsigned)((k + 7) / 8), (unsigned)n);
  auto st = at::cuda::getCurrentCUDAStream();
  const auto dt = static_cast<at::ScalarType>(dtype);
  BDION_D2_DISPATCH(dt, T, {
    gather_decay_kernel<T><<<grid, 256, 0, st>>>(ptrs.data_ptr<int64_t>(), (int)cols, ld, idx.data_ptr<int64_t>(),
                                                k, (float)decay,
                                                reinterpret_cast<__nv_bfloat16*>(sel.data_ptr<at::BFloat16>()));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// X_b = keep * X_b - alpha * scatter(U_b) (rows given by pos), every row of every matrix.
void dion2_update(const at::Tensor& ptrs, int64_t rows, int64_t cols, int64_t ld, int64_t dtype,
                  const at::Tensor& pos, const at::Tensor& U, double keep, double alpha) {
  check_ptrs(ptrs);
  const int n = (int)ptrs.numel();
  TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.numel() == n * rows,
              "dion_b200 dion2_update: pos must be a contiguous int32 [n, rows] tensor");
  TORCH_CHECK(U.is_cuda() && U.scalar_type() == at::kBFloat16 && U.is_contiguous() && U.dim() == 3 &&
                  U.size(0) == n && U.size(2) == cols,
              "dion_b200 dion2_update: U must be a contiguous bf16 [n, k, cols] tensor");
  c10::cuda::CUDAGuard guard(ptrs.device());
  const dim3 grid((unsigned)((rows + 7) / 8), (unsigned)n);
  auto st = at::cuda::getCurrentCUDAStream();
  const auto dt = static_cast<at::ScalarType>(dtype);
  BDION_D2_DISPATCH(dt, T, {
    sparse_update_kernel<T><<<grid, 256, 0, st>>>(ptrs.data_ptr<int64_t>(), (int)rows, (int)cols, ld,
                                                 pos.data_ptr<int>(),
                                                 reinterpret_cast<const __nv_bfloat16*>(U.data_ptr<at::BFloat16>()),
                                                 (int)U.size(1), (float)keep, (float)alpha);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace bdion

// Dion power-iteration helpers (fp32 math):
//   * multi-tensor momentum accumulate M += G with a per-matrix "not all
//     zero" flag (max |M|), feeding the all-zero/NaN guard;
//   * the guard itself: P = nan_to_num(P) * nz ; R = nan_to_num(R) * nz + Q0 * !nz
//   * per-column sum of squares of a batch of (rows x r) matrices, and the
//     column normalisation Q = R / (sqrt(sumsq) + eps) written in Q's dtype.
// Reference behaviour: ada_dion/optim/adadion_v2.py:1795-1869
// (fix_all_zero_or_nan, local_column_sum_sq, column_normalize).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

constexpr int kMax = 48;
constexpr int kChunk = 16384;
constexpr int kThreads = 256;

struct AddArgs {
  int n;
  void* m[kMax];
  const void* g[kMax];
  int64_t numel[kMax];
  int chunk_start[kMax + 1];
};

__device__ __forceinline__ float nan0(float v) { return (v != v) ? 0.f : (isinf(v) ? copysignf(3.402823466e38f, v) : v); }

// 4-element vector load / store of fp32 (16 bytes) or bf16 (8 bytes), as fp32
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 x = *reinterpret_cast<const float4*>(p);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&x.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&x.y);
  v[0] = __low2float(lo); v[1] = __high2float(lo); v[2] = __low2float(hi); v[3] = __high2float(hi);
}
__device__ __forceinline__ void store4(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(v[2], v[3]);
  uint2 x;
  x.x = *reinterpret_cast<const uint32_t*>(&lo);
  x.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = x;
}

template <typename MT, typename GT>
__global__ void __launch_bounds__(kThreads) momentum_add_kernel(AddArgs a, float* partial_max) {
  __shared__ float sh[32];
  const int blk = blockIdx.x;
  int t = 0;
  while (t + 1 < a.n && a.chunk_start[t + 1] <= blk) ++t;
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  MT* M = reinterpret_cast<MT*>(a.m[t]);
  const GT* G = reinterpret_cast<const GT*>(a.g[t]);
  float mx = 0.f;
  // four elements a thread per access when both rows of storage allow it
  // (16-byte fp32 / 8-byte bf16 groups); chunks start at multiples of 4
  const bool vec = (a.numel[t] % 4 == 0) && (reinterpret_cast<uintptr_t>(M) % (4 * sizeof(MT)) == 0) &&
                   (reinterpret_cast<uintptr_t>(G) % (4 * sizeof(GT)) == 0);
  if (vec) {
    for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * kThreads) {
      float m4[4], g4[4];
      load4(M + i, m4);
      load4(G + i, g4);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        m4[e] += g4[e];
        mx = fmaxf(mx, fabsf(m4[e]) + (m4[e] != m4[e] ? 1.f : 0.f));
      }
      store4(M + i, m4);
    }
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) {
      const float v = to_f<MT>(M[i]) + to_f<GT>(G[i]);
      M[i] = from_f<MT>(v);
      mx = fmaxf(mx, fabsf(v) + (v != v ? 1.f : 0.f));
    }
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) r = fmaxf(r, sh[i]);
    partial_max[blk] = r;
  }
}

__global__ void finalize_nz_kernel(AddArgs a, const float* partial_max, float* nz) {
  const int t = blockIdx.x;
  float r = 0.f;
  for (int b = a.chunk_start[t] + threadIdx.x; b < a.chunk_start[t + 1]; b += blockDim.x) r = fmaxf(r, partial_max[b]);
  for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffff, r, o));
  if (threadIdx.x == 0) nz[t] = r > 0.f ? 1.f : 0.f;
}

// P: [b, pn] , R: [b, rn], Q0: [b, rn] (may differ in dtype: QT), nz: [b]
template <typename QT>
__global__ void fixup_kernel(float* P, int64_t pn, float* R, const QT* Q0, int64_t rn, const float* nz) {
  const int b = blockIdx.y;
  const bool keep = nz[b] != 0.f;
  float* Pb = P + (int64_t)b * pn;
  float* Rb = R + (int64_t)b * rn;
  const QT* Qb = Q0 + (int64_t)b * rn;
  // kept matrices are read and rewritten only where a value is not finite
  // (normally nothing is written); dropped ones take P = 0, R = Q0
  const bool vec = pn % 4 == 0 && rn % 4 == 0 && reinterpret_cast<uintptr_t>(Pb) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(Rb) % 16 == 0 && reinterpret_cast<uintptr_t>(Qb) % (4 * sizeof(QT)) == 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    for (int64_t i = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x); i < max(pn, rn); i += 4 * stride) {
      if (i < pn) {
        float v[4];
        if (keep) {
          load4(Pb + i, v);
          if (!(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3]))) {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = nan0(v[e]);
            store4(Pb + i, v);
          }
        } else {
          v[0] = v[1] = v[2] = v[3] = 0.f;
          store4(Pb + i, v);
        }
      }
      if (i < rn) {
        float v[4];
        if (keep) {
          load4(Rb + i, v);
          if (!(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3]))) {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = nan0(v[e]);
            store4(Rb + i, v);
          }
        } else {
          load4(Qb + i, v);
          store4(Rb + i, v);
        }
      }
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < max(pn, rn); i += stride) {
    if (i < pn) Pb[i] = keep ? nan0(Pb[i]) : 0.f;
    if (i < rn) Rb[i] = keep ? nan0(Rb[i]) : to_f<QT>(Qb[i]);
  }
}

// column sum of squares: R [b, rows, r] row-major -> partial [b, chunks, r]
constexpr int kRowsPerChunk = 256;
constexpr int kRowsPerChunk4 = 32;  // vector kernel: more blocks in flight
__global__ void col_sumsq_kernel(const float* R, int rows, int r, float* partial, int chunks) {
  const int b = blockIdx.z, ch = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= r) return;
  const float* Rb = R + (int64_t)b * rows * r;
  const int r0 = ch * kRowsPerChunk, r1 = min(rows, r0 + kRowsPerChunk);
  float s = 0.f;
  for (int i = r0; i < r1; ++i) {
    const float v = Rb[(int64_t)i * r + c];
    s += v * v;
  }
  partial[((int64_t)b * chunks + ch) * r + c] = s;
}

// 4 columns per thread (float4), 8 rows of loads in flight
__global__ void col_sumsq4_kernel(const float* R, int rows, int r, float* partial, int chunks) {
  const int b = blockIdx.z, ch = blockIdx.y;
  const int c4 = blockIdx.x * blockDim.x + threadIdx.x;
  const int r4 = r / 4;
  if (c4 >= r4) return;
  const float4* Rb = reinterpret_cast<const float4*>(R + (int64_t)b * rows * r) + c4;
  const int r0 = ch * kRowsPerChunk4, r1 = min(rows, r0 + kRowsPerChunk4);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  int i = r0;
  for (; i + 8 <= r1; i += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = Rb[(int64_t)(i + u) * r4];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      s.x += v[u].x * v[u].x;
      s.y += v[u].y * v[u].y;
      s.z += v[u].z * v[u].z;
      s.w += v[u].w * v[u].w;
    }
  }
  for (; i < r1; ++i) {
    const float4 v = Rb[(int64_t)i * r4];
    s.x += v.x * v.x;
    s.y += v.y * v.y;
    s.z += v.z * v.z;
    s.w += v.w * v.w;
  }
  reinterpret_cast<float4*>(partial + ((int64_t)b * chunks + ch) * r)[c4] = s;
}

// Q = R / (sqrt(sumsq) + eps): each thread owns 4 columns (one reciprocal
// each) and walks kNormRows rows; Q rows 16-byte (fp32) / 8-byte (bf16) aligned
constexpr int kNormRows = 32;
template <typename QT>
__global__ void col_normalize4_kernel(const float* R, const float* sumsq, int rows, int r, float eps, QT* Q,
                                      int64_t q_bstride, int64_t q_ld) {
  const int b = blockIdx.z;
  const int r4 = r / 4;
  const int c4 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c4 >= r4) return;
  const float4 ss = reinterpret_cast<const float4*>(sumsq + (int64_t)b * r)[c4];
  const float i0 = 1.f / (sqrtf(ss.x) + eps), i1 = 1.f / (sqrtf(ss.y) + eps), i2 = 1.f / (sqrtf(ss.z) + eps),
              i3 = 1.f / (sqrtf(ss.w) + eps);
  const float4* Rb = reinterpret_cast<const float4*>(R + (int64_t)b * rows * r) + c4;
  QT* Qb = Q + (int64_t)b * q_bstride + 4 * c4;
  const int row0 = blockIdx.y * kNormRows, row1 = min(rows, row0 + kNormRows);
#pragma unroll 4
  for (int row = row0; row < row1; ++row) {
    const float4 v = Rb[(int64_t)row * r4];
    QT* q = Qb + (int64_t)row * q_ld;
    if constexpr (sizeof(QT) == 4) {
      *reinterpret_cast<float4*>(q) = make_float4(v.x * i0, v.y * i1, v.z * i2, v.w * i3);
    } else {
      __nv_bfloat162 h[2] = {__floats2bfloat162_rn(v.x * i0, v.y * i1), __floats2bfloat162_rn(v.z * i2, v.w * i3)};
      *reinterpret_cast<uint2*>(q) = *reinterpret_cast<uint2*>(h);
    }
  }
}

__global__ void col_sumsq_finalize(const float* partial, int chunks, int r, int batch, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)batch * r) return;
  const int b = (int)(i / r), c = (int)(i % r);
  float s = 0.f;
  for (int ch = 0; ch < chunks; ++ch) s += partial[((int64_t)b * chunks + ch) * r + c];
  out[i] = s;
}

template <typename QT>
__global__ void col_normalize_kernel(const float* R, const float* sumsq, int rows, int r, float eps, QT* Q,
                                     int64_t q_bstride, int64_t q_ld) {
  const int b = blockIdx.z;
  const int64_t total = (int64_t)rows * r;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / r), c = (int)(i % r);
    const float inv = 1.f / (sqrtf(sumsq[(int64_t)b * r + c]) + eps);
    Q[(int64_t)b * q_bstride + (int64_t)row * q_ld + c] = from_f<QT>(R[(int64_t)b * total + i] * inv);
  }
}

#define DISPATCH_FB(dt, T, ...)                           \
  if ((dt) == at::kFloat) {                               \
    using T = float;                                      \
    __VA_ARGS__                                           \
  } else if ((dt) == at::kBFloat16) {                     \
    using T = __nv_bfloat16;                              \
    __VA_ARGS__                                           \
  } else {                                                \
    TORCH_CHECK(false, "dion_b200: fp32 or bf16 expected"); \
  }

}  // namespace

void dion_momentum_add(const std::vector<at::Tensor>& M, const std::vector<at::Tensor>& G, at::Tensor& nz) {
  if (M.empty()) return;
  c10::cuda::CUDAGuard guard(M[0].device());
  auto s = at::cuda::getCurrentCUDAStream();
  for (size_t b0 = 0; b0 < M.size(); b0 += kMax) {
    const size_t e = std::min(M.size(), b0 + kMax);
    AddArgs a{};
    a.n = (int)(e - b0);
    int chunks = 0;
    for (size_t i = b0; i < e; ++i) {
      TORCH_CHECK(M[i].is_contiguous() && G[i].is_contiguous() && M[i].numel() == G[i].numel(),
                  "dion_b200 momentum_add: contiguous same-size tensors expected");
      a.m[i - b0] = M[i].data_ptr();
      a.g[i - b0] = G[i].data_ptr();
      a.numel[i - b0] = M[i].numel();
      a.chunk_start[i - b0] = chunks;
      chunks += (int)((M[i].numel() + kChunk - 1) / kChunk);
    }
    a.chunk_start[a.n] = chunks;
    auto part = at::empty({chunks}, M[0].options().dtype(at::kFloat));
    DISPATCH_FB(M[0].scalar_type(), MT, DISPATCH_FB(G[0].scalar_type(), GT, {
                  momentum_add_kernel<MT, GT><<<chunks, kThreads, 0, s>>>(a, part.data_ptr<float>());
                }));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    finalize_nz_kernel<<<a.n, 32, 0, s>>>(a, part.data_ptr<float>(), nz.data_ptr<float>() + b0);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
  }
}

void dion_fixup(at::Tensor& P, at::Tensor& R, const at::Tensor& Q0, const at::Tensor& nz) {
  TORCH_CHECK(P.is_contiguous() && R.is_contiguous() && Q0.is_contiguous() && P.scalar_type() == at::kFloat &&
                  R.scalar_type() == at::kFloat,
              "dion_b200 fixup: contiguous fp32 P/R expected");
  c10::cuda::CUDAGuard guard(P.device());
  const int b = (int)P.size(0);
  if (b == 0 || P.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  const int64_t pn = P.numel() / b, rn = R.numel() / b;
  dim3 grid((unsigned)std::min<int64_t>((std::max(pn, rn) + 255) / 256, 1024), b);
  auto s = at::cuda::getCurrentCUDAStream();
  DISPATCH_FB(Q0.scalar_type(), QT, {
    fixup_kernel<QT><<<grid, 256, 0, s>>>(P.data_ptr<float>(), pn, R.data_ptr<float>(),
                                          reinterpret_cast<const QT*>(Q0.data_ptr()), rn, nz.data_ptr<float>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

void col_sumsq(const at::Tensor& R, at::Tensor& out) {
  TORCH_CHECK(R.dim() == 3 && R.is_contiguous() && R.scalar_type() == at::kFloat, "dion_b200 col_sumsq: [b,rows,r] fp32");
  c10::cuda::CUDAGuard guard(R.device());
  const int b = (int)R.size(0), rows = (int)R.size(1), r = (int)R.size(2);
  if (b == 0 || R.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  const bool vec4 = r % 4 == 0;
  const int rows_per_chunk = vec4 ? kRowsPerChunk4 : kRowsPerChunk;
  const int chunks = (rows + rows_per_chunk - 1) / rows_per_chunk;
  auto part = at::empty({b, chunks, r}, R.options());
  auto s = at::cuda::getCurrentCUDAStream();
  if (vec4) {
    dim3 grid((r / 4 + 127) / 128, chunks, b);
    col_sumsq4_kernel<<<grid, 128, 0, s>>>(R.data_ptr<float>(), rows, r, part.data_ptr<float>(), chunks);
  } else {
    dim3 grid((r + 127) / 128, chunks, b);
    col_sumsq_kernel<<<grid, 128, 0, s>>>(R.data_ptr<float>(), rows, r, part.data_ptr<float>(), chunks);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  const int64_t tot = (int64_t)b * r;
  col_sumsq_finalize<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(part.data_ptr<float>(), chunks, r, b,
                                                                     out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// Q (any [b, rows, r] view with unit column stride, fp32 or bf16) = R / (sqrt(sumsq) + eps)
void col_normalize(const at::Tensor& R, const at::Tensor& sumsq, double eps, at::Tensor& Q) {
  TORCH_CHECK(R.dim() == 3 && R.is_contiguous() && R.scalar_type() == at::kFloat, "dion_b200 col_normalize: R fp32");
  TORCH_CHECK(Q.dim() == 3 && Q.stride(2) == 1 && Q.size(1) == R.size(1) && Q.size(2) == R.size(2),
              "dion_b200 col_normalize: Q shape");
  c10::cuda::CUDAGuard guard(R.device());
  const int b = (int)R.size(0), rows = (int)R.size(1), r = (int)R.size(2);
  if (b == 0 || R.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  const int64_t total = (int64_t)rows * r;
  auto s = at::cuda::getCurrentCUDAStream();
  const int qsz = (int)Q.element_size();
  const bool vec = r % 4 == 0 && reinterpret_cast<uintptr_t>(Q.data_ptr()) % (4 * qsz) == 0 &&
                   (Q.stride(1) * qsz) % (4 * qsz) == 0 && (Q.stride(0) * qsz) % (4 * qsz) == 0 &&
                   reinterpret_cast<uintptr_t>(R.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(sumsq.data_ptr()) % 16 == 0;
  if (vec) {
    dim3 grid((unsigned)((r / 4 + 127) / 128), (unsigned)((rows + kNormRows - 1) / kNormRows), (unsigned)b);
    DISPATCH_FB(Q.scalar_type(), QT, {
      col_normalize4_kernel<QT><<<grid, 128, 0, s>>>(R.data_ptr<float>(), sumsq.data_ptr<float>(), rows, r,
                                                     (float)eps, reinterpret_cast<QT*>(Q.data_ptr()), Q.stride(0),
                                                     Q.stride(1));
    });
  } else {
    dim3 grid((unsigned)std::min<int64_t>((total + 255) / 256, 2048), 1, b);
    DISPATCH_FB(Q.scalar_type(), QT, {
      col_normalize_kernel<QT><<<grid, 256, 0, s>>>(R.data_ptr<float>(), sumsq.data_ptr<float>(), rows, r,
                                                    (float)eps, reinterpret_cast<QT*>(Q.data_ptr()), Q.stride(0),
                                                    Q.stride(1));
    });
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// ---------------------------------------------------------------------------
// Adaptive-rank statistic (AdaDionV2): entropy effective rank of the column
// norms of R over each matrix's active columns,
//   s_i = sqrt(max(sumsq_i, 0)) + 1e-12 (i < r_b),  p_i = s_i / (sum s + 1e-12),
//   erank_b = exp(-sum_i p_i log(p_i + 1e-12)).
// One block per matrix; the result stays on the device (the host reads all
// matrices of a shape group with one copy).
namespace {
__device__ __forceinline__ float block_sum256(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  t = red[0];
  __syncthreads();
  return t;
}

__global__ void erank_kernel(const float* __restrict__ sumsq, int width, const int64_t* __restrict__ slots,
                             const int* __restrict__ ranks, float* __restrict__ out) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const float* row = sumsq + slots[m] * (int64_t)width;
  const int r = min(ranks[m], width);
  float s = 0.f;
  for (int i = threadIdx.x; i < r; i += blockDim.x) s += sqrtf(fmaxf(row[i], 0.f)) + 1e-12f;
  const float total = block_sum256(s, red) + 1e-12f;
  float h = 0.f;
  for (int i = threadIdx.x; i < r; i += blockDim.x) {
    const float pr = (sqrtf(fmaxf(row[i], 0.f)) + 1e-12f) / total;
    h -= pr * logf(pr + 1e-12f);
  }
  h = block_sum256(h, red);
  if (threadIdx.x == 0) out[m] = expf(h);
}
}  // namespace

// sumsq [b, width] fp32; slots [n] int64 (rows of sumsq); ranks [n] int32; out [n] fp32
void effective_rank(const at::Tensor& sumsq, const at::Tensor& slots, const at::Tensor& ranks, at::Tensor& out) {
  TORCH_CHECK(sumsq.dim() == 2 && sumsq.is_contiguous() && sumsq.scalar_type() == at::kFloat,
              "dion_b200 effective_rank: sumsq must be a contiguous [b, width] fp32 tensor");
  TORCH_CHECK(slots.scalar_type() == at::kLong && ranks.scalar_type() == at::kInt && out.scalar_type() == at::kFloat,
              "dion_b200 effective_rank: slots int64, ranks int32, out fp32");
  const int64_t n = slots.numel();
  TORCH_CHECK(ranks.numel() == n && out.numel() == n, "dion_b200 effective_rank: sizes");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(sumsq.device());
  erank_kernel<<<(unsigned)n, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      sumsq.data_ptr<float>(), (int)sumsq.size(1), slots.data_ptr<int64_t>(), ranks.data_ptr<int>(),
      out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace bdion

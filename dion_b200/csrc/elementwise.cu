// Multi-tensor elementwise kernels: Muon momentum (+ per-matrix sum of
// squares for the Newton-Schulz normalisation), the Muon/Dion weight update,
// AdamW and Lion. One launch covers up to kMaxTensors tensors; every block
// owns one fixed-size chunk of one tensor.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

constexpr int kMaxTensors = 48;
constexpr int kChunk = 16384;
constexpr int kThreads = 256;

struct MTArgs {
  int n;
  int total_chunks;
  void* p[4][kMaxTensors];
  int64_t numel[kMaxTensors];
  int chunk_start[kMaxTensors + 1];
};

__device__ __forceinline__ int find_tensor(const MTArgs& a, int blk) {
  int t = 0;
  while (t + 1 < a.n && a.chunk_start[t + 1] <= blk) ++t;
  return t;
}

template <typename T>
__device__ __forceinline__ void ld4(const T* p, int64_t i, float* v);
template <>
__device__ __forceinline__ void ld4<float>(const float* p, int64_t i, float* v) {
  float4 a = *reinterpret_cast<const float4*>(p + i);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
template <>
__device__ __forceinline__ void ld4<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i, float* v) {
  uint2 u = *reinterpret_cast<const uint2*>(p + i);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
template <typename T>
__device__ __forceinline__ void st4(T* p, int64_t i, const float* v);
template <>
__device__ __forceinline__ void st4<float>(float* p, int64_t i, const float* v) {
  *reinterpret_cast<float4*>(p + i) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, const float* v) {
  uint2 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
  h[0] = __floats2bfloat162_rn(v[0], v[1]);
  h[1] = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p + i) = u;
}

// Iterate the chunk [lo, hi) of a tensor in 4-element groups (vector path when
// `vec`), calling f(index, count) with count = 4 or the scalar tail count.
template <typename F>
__device__ __forceinline__ void for_chunk(int64_t lo, int64_t hi, bool vec, F f) {
  if (vec) {
    const int64_t hi4 = lo + ((hi - lo) / 4) * 4;
    for (int64_t i = lo + threadIdx.x * 4; i < hi4; i += kThreads * 4) f(i, 4);
    for (int64_t i = hi4 + threadIdx.x; i < hi; i += kThreads) f(i, 1);
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) f(i, 1);
  }
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x / 32] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < kThreads / 32 ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  }
  return s;  // valid in thread 0
}

// ------------------------------------------------------------ Muon momentum
// M = mu*M + G ; U = nesterov ? mu*M + G : M (bf16) ; partial[blk] = sum U^2
template <typename MT, typename GT>
__global__ void __launch_bounds__(kThreads) muon_momentum_kernel(MTArgs a, float mu, int nesterov, int vec,
                                                                 float* partial) {
  __shared__ float sh[32];
  const int blk = blockIdx.x;
  const int t = find_tensor(a, blk);
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  MT* M = reinterpret_cast<MT*>(a.p[0][t]);
  const GT* G = reinterpret_cast<const GT*>(a.p[1][t]);
  __nv_bfloat16* U = reinterpret_cast<__nv_bfloat16*>(a.p[2][t]);
  float ss = 0.f;
  for_chunk(lo, hi, vec, [&](int64_t i, int cnt) {
    float m[4], g[4], u[4];
    if (cnt == 4) {
      ld4<MT>(M, i, m);
      ld4<GT>(G, i, g);
    } else {
      m[0] = to_f<MT>(M[i]);
      g[0] = to_f<GT>(G[i]);
    }
    for (int k = 0; k < cnt; ++k) {
      m[k] = mu * m[k] + g[k];
      u[k] = nesterov ? mu * m[k] + g[k] : m[k];
    }
    if (cnt == 4) {
      st4<MT>(M, i, m);
      st4<__nv_bfloat16>(U, i, u);
      for (int k = 0; k < 4; ++k) {
        float r = __bfloat162float(__float2bfloat16_rn(u[k]));
        ss += r * r;
      }
    } else {
      M[i] = from_f<MT>(m[0]);
      __nv_bfloat16 r = __float2bfloat16_rn(u[0]);
      U[i] = r;
      float rf = __bfloat162float(r);
      ss += rf * rf;
    }
  });
  float s = block_sum(ss, sh);
  if (threadIdx.x == 0) partial[blk] = s;
}

// Per-tensor reduction of block partials, in a fixed order (deterministic).
// out_sumsq[t] = sum ; out_scale[t] = 1 / (sqrt(sum) + eps)
__global__ void finalize_sumsq_kernel(MTArgs a, const float* partial, float* out_sumsq, float* out_scale,
                                      float eps) {
  __shared__ float sh[32];
  const int t = blockIdx.x;
  float s = 0.f;
  for (int b = a.chunk_start[t] + threadIdx.x; b < a.chunk_start[t + 1]; b += kThreads) s += partial[b];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) {
    if (out_sumsq) out_sumsq[t] = s;
    if (out_scale) out_scale[t] = 1.f / (sqrtf(s) + eps);
  }
}

// ------------------------------------------------------------ sum of squares
template <typename T>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(MTArgs a, int vec, float* partial) {
  __shared__ float sh[32];
  const int blk = blockIdx.x;
  const int t = find_tensor(a, blk);
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  const T* X = reinterpret_cast<const T*>(a.p[0][t]);
  float ss = 0.f;
  for_chunk(lo, hi, vec, [&](int64_t i, int cnt) {
    float x[4];
    if (cnt == 4)
      ld4<T>(X, i, x);
    else
      x[0] = to_f<T>(X[i]);
    for (int k = 0; k < cnt; ++k) ss += x[k] * x[k];
  });
  float s = block_sum(ss, sh);
  if (threadIdx.x == 0) partial[blk] = s;
}

// ------------------------------------------------------------ X = decay*X - lr*U
template <typename XT, typename UT>
__global__ void __launch_bounds__(kThreads) scaled_update_kernel(MTArgs a, float decay, const float* lrs, int vec) {
  const int blk = blockIdx.x;
  const int t = find_tensor(a, blk);
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  XT* X = reinterpret_cast<XT*>(a.p[0][t]);
  const UT* U = reinterpret_cast<const UT*>(a.p[1][t]);
  const float lr = lrs[t];
  for_chunk(lo, hi, vec, [&](int64_t i, int cnt) {
    float x[4], u[4];
    if (cnt == 4) {
      ld4<XT>(X, i, x);
      ld4<UT>(U, i, u);
      for (int k = 0; k < 4; ++k) x[k] = decay * x[k] - lr * u[k];
      st4<XT>(X, i, x);
    } else {
      X[i] = from_f<XT>(decay * to_f<XT>(X[i]) - lr * to_f<UT>(U[i]));
    }
  });
}

// ------------------------------------------------------------ AdamW
template <typename XT, typename GT, typename ST>
__global__ void __launch_bounds__(kThreads) adamw_kernel(MTArgs a, float lr, float beta1, float beta2, float wd,
                                                         float eps, float bc1, float bc2_sqrt, int cautious, int vec) {
  const int blk = blockIdx.x;
  const int t = find_tensor(a, blk);
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  XT* X = reinterpret_cast<XT*>(a.p[0][t]);
  const GT* G = reinterpret_cast<const GT*>(a.p[1][t]);
  ST* M = reinterpret_cast<ST*>(a.p[2][t]);
  ST* V = reinterpret_cast<ST*>(a.p[3][t]);
  const float adj_lr = lr / bc1;
  for_chunk(lo, hi, vec, [&](int64_t i, int cnt) {
    float x[4], g[4], m[4], v[4];
    if (cnt == 4) {
      ld4<XT>(X, i, x);
      ld4<GT>(G, i, g);
      ld4<ST>(M, i, m);
      ld4<ST>(V, i, v);
    } else {
      x[0] = to_f<XT>(X[i]);
      g[0] = to_f<GT>(G[i]);
      m[0] = to_f<ST>(M[i]);
      v[0] = to_f<ST>(V[i]);
    }
    for (int k = 0; k < cnt; ++k) {
      m[k] = m[k] + (1.f - beta1) * (g[k] - m[k]);
      v[k] = v[k] + (1.f - beta2) * (g[k] * g[k] - v[k]);
      const float denom = sqrtf(v[k]) / bc2_sqrt + eps;
      const float upd = m[k] / denom;
      if (cautious) {
        if (upd * x[k] >= 0.f) x[k] -= lr * wd * x[k];
      } else {
        x[k] *= (1.f - lr * wd);
      }
      x[k] -= adj_lr * upd;
    }
    if (cnt == 4) {
      st4<XT>(X, i, x);
      st4<ST>(M, i, m);
      st4<ST>(V, i, v);
    } else {
      X[i] = from_f<XT>(x[0]);
      M[i] = from_f<ST>(m[0]);
      V[i] = from_f<ST>(v[0]);
    }
  });
}

// ------------------------------------------------------------ Lion
template <typename XT, typename GT, typename ST>
__global__ void __launch_bounds__(kThreads) lion_kernel(MTArgs a, float lr, float beta1, float beta2, float wd,
                                                        int cautious, int vec) {
  const int blk = blockIdx.x;
  const int t = find_tensor(a, blk);
  const int64_t lo = (int64_t)(blk - a.chunk_start[t]) * kChunk;
  const int64_t hi = min(a.numel[t], lo + kChunk);
  XT* X = reinterpret_cast<XT*>(a.p[0][t]);
  const GT* G = reinterpret_cast<const GT*>(a.p[1][t]);
  ST* M = reinterpret_cast<ST*>(a.p[2][t]);
  for_chunk(lo, hi, vec, [&](int64_t i, int cnt) {
    float x[4], g[4], m[4];
    if (cnt == 4) {
      ld4<XT>(X, i, x);
      ld4<GT>(G, i, g);
      ld4<ST>(M, i, m);
    } else {
      x[0] = to_f<XT>(X[i]);
      g[0] = to_f<GT>(G[i]);
      m[0] = to_f<ST>(M[i]);
    }
    for (int k = 0; k < cnt; ++k) {
      const float c = m[k] + (1.f - beta1) * (g[k] - m[k]);
      const float u = c > 0.f ? 1.f : (c < 0.f ? -1.f : 0.f);
      m[k] = m[k] + (1.f - beta2) * (g[k] - m[k]);
      if (cautious) {
        if (u * x[k] >= 0.f) x[k] -= lr * wd * x[k];
      } else {
        x[k] *= (1.f - lr * wd);
      }
      x[k] -= lr * u;
    }
    if (cnt == 4) {
      st4<XT>(X, i, x);
      st4<ST>(M, i, m);
    } else {
      X[i] = from_f<XT>(x[0]);
      M[i] = from_f<ST>(m[0]);
    }
  });
}

// ------------------------------------------------------------ host helpers
bool is16(const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; }

// Build launch descriptors for up to kMaxTensors tensors of lists[0..nl).
MTArgs build_args(const std::vector<const std::vector<at::Tensor>*>& lists, size_t begin, size_t end, bool& vec) {
  MTArgs a{};
  a.n = (int)(end - begin);
  int chunks = 0;
  vec = true;
  for (size_t i = begin; i < end; ++i) {
    const int64_t n = (*lists[0])[i].numel();
    a.numel[i - begin] = n;
    a.chunk_start[i - begin] = chunks;
    chunks += (int)((n + kChunk - 1) / kChunk);
    for (size_t l = 0; l < lists.size(); ++l) {
      const at::Tensor& t = (*lists[l])[i];
      TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "dion_b200: multi-tensor inputs must be contiguous CUDA tensors");
      TORCH_CHECK(t.numel() == n, "dion_b200: multi-tensor size mismatch");
      a.p[l][i - begin] = t.data_ptr();
      vec = vec && is16(t);
    }
  }
  a.chunk_start[a.n] = chunks;
  a.total_chunks = chunks;
  return a;
}

template <typename F>
void for_batches(size_t n, F f) {
  for (size_t b = 0; b < n; b += kMaxTensors) f(b, std::min(n, b + kMaxTensors));
}

#define BDION_DISPATCH_FB(dt, T, ...)                                   \
  if ((dt) == at::kFloat) {                                             \
    using T = float;                                                    \
    __VA_ARGS__                                                         \
  } else if ((dt) == at::kBFloat16) {                                   \
    using T = __nv_bfloat16;                                            \
    __VA_ARGS__                                                         \
  } else {                                                              \
    TORCH_CHECK(false, "dion_b200: only fp32 and bf16 tensors are supported"); \
  }

}  // namespace

// M, G: lists of same-size tensors; U: bf16 outputs. Returns nothing; writes
// sumsq[i] and scale[i] = 1/(sqrt(sumsq[i]) + eps) (fp32 device vectors).
void muon_momentum(const std::vector<at::Tensor>& M, const std::vector<at::Tensor>& G,
                   const std::vector<at::Tensor>& U, double mu, bool nesterov, at::Tensor& sumsq, at::Tensor& scale,
                   double eps) {
  TORCH_CHECK(M.size() == G.size() && M.size() == U.size(), "dion_b200 muon_momentum: list sizes differ");
  if (M.empty()) return;
  c10::cuda::CUDAGuard guard(M[0].device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  for_batches(M.size(), [&](size_t b, size_t e) {
    bool vec;
    MTArgs a = build_args({&M, &G, &U}, b, e, vec);
    auto partial = at::empty({a.total_chunks}, M[0].options().dtype(at::kFloat));
    BDION_DISPATCH_FB(M[0].scalar_type(), MT, BDION_DISPATCH_FB(G[0].scalar_type(), GT, {
                        muon_momentum_kernel<MT, GT><<<a.total_chunks, kThreads, 0, s>>>(
                            a, (float)mu, nesterov ? 1 : 0, vec ? 1 : 0, partial.data_ptr<float>());
                      }));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
    finalize_sumsq_kernel<<<a.n, kThreads, 0, s>>>(a, partial.data_ptr<float>(), sumsq.data_ptr<float>() + b,
                                                     scale.data_ptr<float>() + b, (float)eps);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  });
}

void multi_sumsq(const std::vector<at::Tensor>& X, at::Tensor& sumsq) {
  if (X.empty()) return;
  c10::cuda::CUDAGuard guard(X[0].device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  for_batches(X.size(), [&](size_t b, size_t e) {
    bool vec;
    MTArgs a = build_args({&X}, b, e, vec);
    auto partial = at::empty({a.total_chunks}, X[0].options().dtype(at::kFloat));
    BDION_DISPATCH_FB(X[0].scalar_type(), T, {
      sumsq_kernel<T><<<a.total_chunks, kThreads, 0, s>>>(a, vec ? 1 : 0, partial.data_ptr<float>());
    });
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
    finalize_sumsq_kernel<<<a.n, kThreads, 0, s>>>(a, partial.data_ptr<float>(), sumsq.data_ptr<float>() + b,
                                                     nullptr, 0.f);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  });
}

// X[i] = decay * X[i] - lrs[i] * U[i]  (lrs: fp32 device vector)
void scaled_update(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& U, double decay,
                   const at::Tensor& lrs) {
  if (X.empty()) return;
  c10::cuda::CUDAGuard guard(X[0].device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  for_batches(X.size(), [&](size_t b, size_t e) {
    bool vec;
    MTArgs a = build_args({&X, &U}, b, e, vec);
    BDION_DISPATCH_FB(X[0].scalar_type(), XT, BDION_DISPATCH_FB(U[0].scalar_type(), UT, {
                        scaled_update_kernel<XT, UT><<<a.total_chunks, kThreads, 0, s>>>(
                            a, (float)decay, lrs.data_ptr<float>() + b, vec ? 1 : 0);
                      }));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  });
}

void adamw(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& G, const std::vector<at::Tensor>& M,
           const std::vector<at::Tensor>& V, double lr, double beta1, double beta2, double wd, double eps,
           int64_t step, bool cautious) {
  if (X.empty()) return;
  c10::cuda::CUDAGuard guard(X[0].device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const double bc1 = 1.0 - std::pow(beta1, (double)step);
  const double bc2s = std::sqrt(1.0 - std::pow(beta2, (double)step));
  for_batches(X.size(), [&](size_t b, size_t e) {
    bool vec;
    MTArgs a = build_args({&X, &G, &M, &V}, b, e, vec);
    BDION_DISPATCH_FB(X[0].scalar_type(), XT, BDION_DISPATCH_FB(G[0].scalar_type(), GT, BDION_DISPATCH_FB(M[0].scalar_type(), ST, {
                        adamw_kernel<XT, GT, ST><<<a.total_chunks, kThreads, 0, s>>>(
                            a, (float)lr, (float)beta1, (float)beta2, (float)wd, (float)eps, (float)bc1,
                            (float)bc2s, cautious ? 1 : 0, vec ? 1 : 0);
                      })));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  });
}

void lion(const std::vector<at::Tensor>& X, const std::vector<at::Tensor>& G, const std::vector<at::Tensor>& M,
          double lr, double beta1, double beta2, double wd, bool cautious) {
  if (X.empty()) return;
  c10::cuda::CUDAGuard guard(X[0].device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  for_batches(X.size(), [&](size_t b, size_t e) {
    bool vec;
    MTArgs a = build_args({&X, &G, &M}, b, e, vec);
    BDION_DISPATCH_FB(X[0].scalar_type(), XT, BDION_DISPATCH_FB(G[0].scalar_type(), GT, BDION_DISPATCH_FB(M[0].scalar_type(), ST, {
                        lion_kernel<XT, GT, ST><<<a.total_chunks, kThreads, 0, s>>>(
                            a, (float)lr, (float)beta1, (float)beta2, (float)wd, cautious ? 1 : 0, vec ? 1 : 0);
                      })));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  });
}

}  // namespace bdion

// ---------------------------------------------------------------- allocation-free entry point
// bdion_batched_sumsq_noalloc (declared and documented in no_alloc.h) runs the
// same sum-of-squares kernels as multi_sumsq above, with the block partials
// kept in a fixed file-scope device array instead of a freshly allocated
// buffer, so the call allocates no device memory at all.
#include <cstdio>
#include <mutex>

#include "no_alloc.h"

static __device__ __align__(256) float g_noalloc_partials[BDION_NOALLOC_MAX_PARTIALS];

namespace bdion {
namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_scratch[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (looked up once
// per device; the host-side symbol is only a stand-in, never a device address).
float* noalloc_scratch(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_partials) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // reset the runtime's last-error value after the failed lookup
      return nullptr;
    }
    g_noalloc_scratch[dev] = static_cast<float*>(p);
  }
  return g_noalloc_scratch[dev];
}

}  // namespace
}  // namespace bdion

extern "C" __attribute__((visibility("default"))) int bdion_batched_sumsq_noalloc(const void* x, int dtype,
                                                                                  int64_t batch, int64_t numel,
                                                                                  int64_t stride, float* out,
                                                                                  void* stream) {
  using namespace bdion;
  if (x == nullptr || out == nullptr || batch < 1 || numel < 1 || stride < numel || (dtype != 0 && dtype != 1))
    return BDION_NOALLOC_BAD_ARGUMENT;
  const int64_t chunks_per = (numel + kChunk - 1) / kChunk;
  if (chunks_per > BDION_NOALLOC_MAX_PARTIALS || batch > BDION_NOALLOC_MAX_PARTIALS / chunks_per) {
    std::fprintf(stderr,
                 "bdion_batched_sumsq_noalloc: %lld tensors of %lld elements need %lld partial sums, more than the "
                 "fixed scratch capacity of %d\n",
                 (long long)batch, (long long)numel, (long long)(batch * chunks_per), BDION_NOALLOC_MAX_PARTIALS);
    return BDION_NOALLOC_TOO_LARGE;
  }
  // an error left by earlier work is reported as such and stays set (peek, not get)
  if (cudaPeekAtLastError() != cudaSuccess) return BDION_NOALLOC_PENDING_ERROR;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return BDION_NOALLOC_SETUP_FAILED;
  float* scratch = noalloc_scratch(dev);
  if (scratch == nullptr) return BDION_NOALLOC_SETUP_FAILED;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int esz = dtype == 0 ? 4 : 2;
  const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && (stride * esz) % 16 == 0;
  int64_t used = 0;  // each launch group writes its own slice of the scratch array
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxTensors) {
    const int n = (int)std::min<int64_t>(kMaxTensors, batch - b0);
    MTArgs a{};
    a.n = n;
    int chunks = 0;
    for (int i = 0; i < n; ++i) {
      a.p[0][i] = const_cast<char*>(static_cast<const char*>(x)) + (b0 + i) * stride * esz;
      a.numel[i] = numel;
      a.chunk_start[i] = chunks;
      chunks += (int)chunks_per;
    }
    a.chunk_start[n] = chunks;
    a.total_chunks = chunks;
    float* part = scratch + used;
    if (dtype == 0)
      sumsq_kernel<float><<<chunks, kThreads, 0, s>>>(a, vec ? 1 : 0, part);
    else
      sumsq_kernel<__nv_bfloat16><<<chunks, kThreads, 0, s>>>(a, vec ? 1 : 0, part);
    if (cudaPeekAtLastError() != cudaSuccess) return BDION_NOALLOC_LAUNCH_FAILED;
    finalize_sumsq_kernel<<<n, kThreads, 0, s>>>(a, part, out + b0, nullptr, 0.f);
    if (cudaPeekAtLastError() != cudaSuccess) return BDION_NOALLOC_LAUNCH_FAILED;
    note_launch(2);
    used += chunks;
  }
  return BDION_NOALLOC_OK;
}

// Memory-bound model kernels: RMSNorm (fwd/bwd), rotary embedding, SwiGLU
// (fwd/bwd) and a fused softmax-cross-entropy forward+backward. All bf16 in
// and out with fp32 math; every kernel reads and writes each tensor once
// (RMSNorm re-reads its row from L1).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

// ------------------------------------------------------------ RMSNorm
// one warp per row; D % 8 == 0
template <typename WT>
__global__ void rms_fwd_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int R, int D, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= R) return;
  const __nv_bfloat16* xr = x + (int64_t)row * D;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[row] = r;
  __nv_bfloat16* yr = y + (int64_t)row * D;
  for (int c = lane * 8; c < D; c += 256) {
    float v[8], wv[8];
    load8(xr + c, v);
    load8(w + c, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * r * wv[i];
    store8(yr + c, v);
  }
}

// Same, for D = NC*256: the row stays in registers between the sum of
// squares and the scaling, so x is read from memory once.
template <typename WT, int NC>
__global__ void rms_fwd_reg_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int R, float eps) {
  constexpr int D = NC * 256;
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= R) return;
  const __nv_bfloat16* xr = x + (int64_t)row * D;
  float v[NC][8];
#pragma unroll
  for (int k = 0; k < NC; ++k) load8(xr + k * 256 + lane * 8, v[k]);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k)
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[row] = r;
  __nv_bfloat16* yr = y + (int64_t)row * D;
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    float wv[8];
    load8(w + k * 256 + lane * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[k][i] = v[k][i] * r * wv[i];
    store8(yr + k * 256 + lane * 8, v[k]);
  }
}

// gx = r*w*gy - x * r^3/D * sum(gy*w*x); partial gw[blk, :] += gy*x*r over this block's rows
template <typename WT>
__global__ void rms_bwd_kernel(const __nv_bfloat16* __restrict__ gy, const __nv_bfloat16* __restrict__ x,
                               const WT* __restrict__ w, const float* __restrict__ rstd,
                               __nv_bfloat16* __restrict__ gx, float* __restrict__ gw_part, int R, int D,
                               int rows_per_block) {
  extern __shared__ float sgw[];  // [warps][D]
  const int warps = blockDim.x / 32;
  const int wid = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* my = sgw + (size_t)wid * D;
  for (int c = lane; c < D; c += 32) my[c] = 0.f;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  for (int row = r0 + wid; row < r1; row += warps) {
    const __nv_bfloat16* xr = x + (int64_t)row * D;
    const __nv_bfloat16* gr = gy + (int64_t)row * D;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      float xv[8], gv[8], wv[8];
      load8(xr + c, xv);
      load8(gr + c, gv);
      load8(w + c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dot += gv[i] * wv[i] * xv[i];
        my[c + i] += gv[i] * xv[i] * r;
      }
    }
    dot = warp_sum(dot);
    const float k = r * r * r * dot / D;
    __nv_bfloat16* gxr = gx + (int64_t)row * D;
    for (int c = lane * 8; c < D; c += 256) {
      float xv[8], gv[8], wv[8], o[8];
      load8(xr + c, xv);
      load8(gr + c, gv);
      load8(w + c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = r * wv[i] * gv[i] - xv[i] * k;
      store8(gxr + c, o);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < warps; ++i) s += sgw[(size_t)i * D + c];
    gw_part[(int64_t)blockIdx.x * D + c] = s;
  }
}

// ------------------------------------------------------------ RoPE
// x: [b, s, h, d] contiguous; table [S, d/2, 2] (cos, sin); interleaved pairs
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const float* __restrict__ tab, __nv_bfloat16* __restrict__ qo,
                            __nv_bfloat16* __restrict__ ko, int64_t nq_pairs, int64_t nk_pairs, int S, int hq,
                            int hk, int half, float sign) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  int64_t p;
  int h;
  if (i < nq_pairs) {
    src = q; dst = qo; p = i; h = hq;
  } else if (i < nq_pairs + nk_pairs) {
    src = k; dst = ko; p = i - nq_pairs; h = hk;
  } else {
    return;
  }
  const int j = (int)(p % half);
  const int64_t pos = (p / half / h) % S;
  const float c = tab[(pos * half + j) * 2];
  const float s = sign * tab[(pos * half + j) * 2 + 1];
  const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(src)[p];
  const float2 f = __bfloat1622float2(v);
  reinterpret_cast<__nv_bfloat162*>(dst)[p] = __floats2bfloat162_rn(f.x * c - f.y * s, f.x * s + f.y * c);
}


// Register-accumulating variant for D = NC * 256: each lane owns the columns
// {lane*8 + c*256 + i}, keeps its share of the weight gradient in registers
// across all rows of the block and writes one partial row at the end.
template <typename WT, int NC>
__global__ void __launch_bounds__(128) rms_bwd_reg_kernel(const __nv_bfloat16* __restrict__ gy,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const WT* __restrict__ w, const float* __restrict__ rstd,
                                                          __nv_bfloat16* __restrict__ gx,
                                                          float* __restrict__ gw_part, int R, int rows_per_block) {
  constexpr int D = NC * 256;
  extern __shared__ float red[];  // [4][D] partial weight gradients, one row per warp
  const int wid = threadIdx.x / 32, lane = threadIdx.x % 32;
  float acc[NC][8];
  float wv[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    load8(w + c * 256 + lane * 8, wv[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  for (int row = r0 + wid; row < r1; row += 4) {
    const __nv_bfloat16* xr = x + (int64_t)row * D;
    const __nv_bfloat16* gr = gy + (int64_t)row * D;
    const float r = rstd[row];
    float xv[NC][8], gv[NC][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      load8(xr + c * 256 + lane * 8, xv[c]);
      load8(gr + c * 256 + lane * 8, gv[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dot += gv[c][i] * wv[c][i] * xv[c][i];
        acc[c][i] += gv[c][i] * xv[c][i] * r;
      }
    }
    dot = warp_sum(dot);
    const float k = r * r * r * dot / D;
    __nv_bfloat16* gxr = gx + (int64_t)row * D;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = r * wv[c][i] * gv[c][i] - xv[c][i] * k;
      store8(gxr + c * 256 + lane * 8, o);
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[wid * D + c * 256 + lane * 8 + i] = acc[c][i];
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += 128)
    gw_part[(int64_t)blockIdx.x * D + col] = red[col] + red[D + col] + red[2 * D + col] + red[3 * D + col];
}

// One CTA per group of rows, D / 8 threads: thread t owns columns
// [8t, 8t + 8) of every row, so the weight and its share of the weight
// gradient stay in 16 registers whatever D is (the warp-per-row variant above
// keeps 4 x D / 32 values per lane and runs out of registers at D = 2048).
// The row's dot product is one block reduction per row; the per-warp
// partials are double-buffered so one barrier per row suffices.
// gres (optional): a gradient added to gx in the same pass (the residual
// branch of a fused add + norm).
template <typename WT>
__global__ void __launch_bounds__(1024) rms_bwd_row_kernel(const __nv_bfloat16* __restrict__ gy,
                                                           const __nv_bfloat16* __restrict__ x,
                                                           const WT* __restrict__ w, const float* __restrict__ rstd,
                                                           __nv_bfloat16* __restrict__ gx,
                                                           float* __restrict__ gw_part, int R, int D,
                                                           int rows_per_block,
                                                           const __nv_bfloat16* __restrict__ gres) {
  __shared__ float wsum[2][32];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int col = t * 8;
  float wv[8], acc[8];
  load8(w + col, wv);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  int buf = 0;
  for (int row = r0; row < r1; ++row) {
    float xv[8], gv[8];
    load8(x + (int64_t)row * D + col, xv);
    load8(gy + (int64_t)row * D + col, gv);
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dot += gv[i] * wv[i] * xv[i];
      acc[i] += gv[i] * xv[i] * r;
    }
    dot = warp_sum(dot);
    if (lane == 0) wsum[buf][wid] = dot;
    __syncthreads();
    float tot = 0.f;
    for (int q = 0; q < nw; ++q) tot += wsum[buf][q];
    buf ^= 1;
    const float k = r * r * r * tot / D;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = r * wv[i] * gv[i] - xv[i] * k;
    if (gres != nullptr) {
      float rv[8];
      load8(gres + (int64_t)row * D + col, rv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += rv[i];
    }
    store8(gx + (int64_t)row * D + col, o);
  }
  float* gp = gw_part + (int64_t)blockIdx.x * D + col;
#pragma unroll
  for (int i = 0; i < 8; ++i) gp[i] = acc[i];
}

// h = x + a (rounded to bf16, as the unfused add) and y = h * rstd(h) * w,
// one CTA of D / 8 threads per group of rows (thread t: columns [8t, 8t+8)).
template <typename WT>
__global__ void __launch_bounds__(1024) add_rms_fwd_row_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ a,
                                                               const WT* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ h,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ rstd, int R, int D,
                                                               int rows_per_block, float eps) {
  __shared__ float wsum[2][32];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int col = t * 8;
  float wv[8];
  load8(w + col, wv);
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  int buf = 0;
  for (int row = r0; row < r1; ++row) {
    float xv[8], av[8];
    load8(x + (int64_t)row * D + col, xv);
    load8(a + (int64_t)row * D + col, av);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i] = __bfloat162float(__float2bfloat16_rn(xv[i] + av[i]));
      ss += xv[i] * xv[i];
    }
    store8(h + (int64_t)row * D + col, xv);
    ss = warp_sum(ss);
    if (lane == 0) wsum[buf][wid] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int q = 0; q < nw; ++q) tot += wsum[buf][q];
    buf ^= 1;
    const float r = rsqrtf(tot / D + eps);
    if (t == 0) rstd[row] = r;
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = xv[i] * r * wv[i];
    store8(y + (int64_t)row * D + col, xv);
  }
}

// RoPE over 8 consecutive elements (4 interleaved pairs) per thread; one
// table row (cos, sin per pair) per position.
__global__ void rope8_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                             const float2* __restrict__ tab, __nv_bfloat16* __restrict__ qo,
                             __nv_bfloat16* __restrict__ ko, int64_t nq8, int64_t nk8, int S, int hq, int hk,
                             int half, float sign) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  int64_t v;
  int h;
  if (i < nq8) {
    src = q; dst = qo; v = i; h = hq;
  } else if (i < nq8 + nk8) {
    src = k; dst = ko; v = i - nq8; h = hk;
  } else {
    return;
  }
  const int per_row = half / 4;              // 8-element groups per head row
  const int64_t row = v / per_row;           // (b, s, head)
  const int j0 = (int)(v - row * per_row) * 4;
  const int pos = (int)((row / h) % S);
  float x[8];
  load8(src + v * 8, x);
  const float2* t = tab + (int64_t)pos * half + j0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 cs = t[p];
    const float c = cs.x, s = sign * cs.y;
    const float a = x[2 * p], b = x[2 * p + 1];
    x[2 * p] = a * c - b * s;
    x[2 * p + 1] = a * s + b * c;
  }
  store8(dst + v * 8, x);
}

// RoPE with one CTA per (batch, position): the position and its table row
// are fixed for the CTA, so no thread divides a 64-bit index (the per-element
// variant above spends more time on index division than on memory). Thread
// t handles 8-element groups t, t + blockDim, ... of the position's q heads
// then k heads.
__global__ void __launch_bounds__(128) rope_pos_kernel(const __nv_bfloat16* __restrict__ q,
                                                       const __nv_bfloat16* __restrict__ k,
                                                       const float2* __restrict__ tab, __nv_bfloat16* __restrict__ qo,
                                                       __nv_bfloat16* __restrict__ ko, int S, int hq, int hk, int half,
                                                       float sign) {
  const int bs = blockIdx.x;  // b * S + s
  const int pos = bs % S;
  const int per_head = half / 4;  // 8-element groups per head
  const int nq = hq * per_head, nk = hk * per_head;
  const float2* trow = tab + (int64_t)pos * half;
  const int64_t qbase = (int64_t)bs * hq * half * 2, kbase = (int64_t)bs * hk * half * 2;
  for (int g = threadIdx.x; g < nq + nk; g += blockDim.x) {
    const bool isq = g < nq;
    const int gg = isq ? g : g - nq;
    const int j0 = (gg % per_head) * 4;
    const __nv_bfloat16* src = (isq ? q + qbase : k + kbase) + (int64_t)gg * 8;
    __nv_bfloat16* dst = (isq ? qo + qbase : ko + kbase) + (int64_t)gg * 8;
    float x[8];
    load8(src, x);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 cs = trow[j0 + p];
      const float c = cs.x, sn = sign * cs.y;
      const float a = x[2 * p], b = x[2 * p + 1];
      x[2 * p] = a * c - b * sn;
      x[2 * p + 1] = a * sn + b * c;
    }
    store8(dst, x);
  }
}

// ------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                  __nv_bfloat16* __restrict__ o, int64_t n8) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float av[8], bv[8], ov[8];
    load8(a + i * 8, av);
    load8(b + i * 8, bv);
#pragma unroll
    for (int t = 0; t < 8; ++t) ov[t] = av[t] * sigmoidf_(av[t]) * bv[t];
    store8(o + i * 8, ov);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ a,
                                  const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ ga,
                                  __nv_bfloat16* __restrict__ gb, int64_t n8) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float gv[8], av[8], bv[8], gav[8], gbv[8];
    load8(g + i * 8, gv);
    load8(a + i * 8, av);
    load8(b + i * 8, bv);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float s = sigmoidf_(av[t]);
      const float silu = av[t] * s;
      gbv[t] = gv[t] * silu;
      gav[t] = gv[t] * bv[t] * (s + silu * (1.f - s));
    }
    store8(ga + i * 8, gav);
    store8(gb + i * 8, gbv);
  }
}

// ------------------------------------------------------------ cross-entropy
// one block per row: lse by an online max/sum pass, then grad = scale*(p - onehot)
constexpr int kCeThreads = 512;
__global__ void __launch_bounds__(kCeThreads) ce_kernel(const __nv_bfloat16* __restrict__ logits,
                                                        const int64_t* __restrict__ labels,
                                                        __nv_bfloat16* __restrict__ grad, float* __restrict__ row_loss,
                                                        int V, float scale) {
  __shared__ float smax[32], ssum[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* lr = logits + (int64_t)row * V;
  float m = -INFINITY, s = 0.f;
  const int V8 = V / 8;
  for (int c = threadIdx.x; c < V8; c += kCeThreads) {
    float v[8];
    load8(lr + c * 8, v);
    float lm = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, v[i]);
    if (lm > m) {
      s *= __expf(m - lm);
      m = lm;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) s += __expf(v[i] - m);
  }
  for (int c = V8 * 8 + threadIdx.x; c < V; c += kCeThreads) {
    const float v = __bfloat162float(lr[c]);
    if (v > m) {
      s *= __expf(m - v);
      m = v;
    }
    s += __expf(v - m);
  }
  // combine (m, s) across the block
  float wm = warp_max(m);
  s = (m == -INFINITY) ? 0.f : s * __expf(m - wm);
  s = warp_sum(s);
  const int wid = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    smax[wid] = wm;
    ssum[wid] = s;
  }
  __syncthreads();
  if (wid == 0) {
    const int nw = kCeThreads / 32;
    float m2 = lane < nw ? smax[lane] : -INFINITY;
    float s2 = lane < nw ? ssum[lane] : 0.f;
    const float gm = warp_max(m2);
    s2 = (m2 == -INFINITY) ? 0.f : s2 * __expf(m2 - gm);
    s2 = warp_sum(s2);
    if (lane == 0) {
      smax[0] = gm;
      ssum[0] = s2;
    }
  }
  __syncthreads();
  const float lse = smax[0] + __logf(ssum[0]);
  const int64_t lab = labels[row];
  if (threadIdx.x == 0) row_loss[row] = lse - __bfloat162float(lr[lab]);
  __nv_bfloat16* gr = grad + (int64_t)row * V;
  for (int c = threadIdx.x; c < V8; c += kCeThreads) {
    float v[8];
    load8(lr + c * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = __expf(v[i] - lse);
      if ((int64_t)(c * 8 + i) == lab) v[i] -= 1.f;
      v[i] *= scale;
    }
    store8(gr + c * 8, v);
  }
  for (int c = V8 * 8 + threadIdx.x; c < V; c += kCeThreads) {
    float v = __expf(__bfloat162float(lr[c]) - lse);
    if (c == lab) v -= 1.f;
    gr[c] = __float2bfloat16_rn(v * scale);
  }
}

}  // namespace

void rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps) {
  const int R = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(D % 8 == 0 && x.is_contiguous() && w.is_contiguous(), "dion_b200 rms_norm: D % 8 and contiguous");
  c10::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int rows_per_blk = 4;
  const int grid = (R + rows_per_blk - 1) / rows_per_blk;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  const int nc = D % 256 == 0 ? D / 256 : 0;
  if (nc == 1 || nc == 2 || nc == 3 || nc == 4 || nc == 8 || nc == 16) {
    auto launch = [&](auto tag_w, auto ncc) {
      using WT = decltype(tag_w);
      constexpr int NC = decltype(ncc)::value;
      rms_fwd_reg_kernel<WT, NC><<<grid, 128, 0, s>>>(xp, reinterpret_cast<const WT*>(w.data_ptr()), yp,
                                                       rstd.data_ptr<float>(), R, (float)eps);
    };
    auto by_nc = [&](auto tag_w) {
      switch (nc) {
        case 1: launch(tag_w, std::integral_constant<int, 1>{}); break;
        case 2: launch(tag_w, std::integral_constant<int, 2>{}); break;
        case 3: launch(tag_w, std::integral_constant<int, 3>{}); break;
        case 4: launch(tag_w, std::integral_constant<int, 4>{}); break;
        case 8: launch(tag_w, std::integral_constant<int, 8>{}); break;
        default: launch(tag_w, std::integral_constant<int, 16>{}); break;
      }
    };
    if (w.scalar_type() == at::kFloat)
      by_nc(float{});
    else
      by_nc(__nv_bfloat16{});
  } else if (w.scalar_type() == at::kFloat)
    rms_fwd_kernel<float><<<grid, 128, 0, s>>>(xp, w.data_ptr<float>(), yp, rstd.data_ptr<float>(), R, D, (float)eps);
  else
    rms_fwd_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
        xp, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), yp, rstd.data_ptr<float>(), R, D, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

void rms_norm_bwd(const at::Tensor& gy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                  at::Tensor& gx, at::Tensor& gw) {
  const int R = (int)x.size(0), D = (int)x.size(1);
  c10::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int warps = 4;
  const size_t smem = (size_t)warps * D * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "dion_b200 rms_norm_bwd: D too large");
  if (D % 256 == 0 && D >= 1024 && D <= 8192) {
    // row-per-CTA variant: D / 8 threads, a few CTAs per SM
    const int threads = D / 8;
    const int per_sm = std::max(1, 2048 / threads);
    const int nblk = std::min(R, sms * per_sm);
    const int rpb = (R + nblk - 1) / nblk;
    auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
    auto gyp = reinterpret_cast<const __nv_bfloat16*>(gy.data_ptr());
    auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    auto gxp = reinterpret_cast<__nv_bfloat16*>(gx.data_ptr());
    if (w.scalar_type() == at::kFloat)
      rms_bwd_row_kernel<float><<<nblk, threads, 0, s>>>(gyp, xp, w.data_ptr<float>(), rstd.data_ptr<float>(), gxp,
                                                         part.data_ptr<float>(), R, D, rpb, nullptr);
    else
      rms_bwd_row_kernel<__nv_bfloat16><<<nblk, threads, 0, s>>>(
          gyp, xp, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(), gxp,
          part.data_ptr<float>(), R, D, rpb, nullptr);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    at::sum_out(gw, part, 0);
    return;
  }
  if (D % 256 == 0 && (D / 256 == 1 || D / 256 == 2 || D / 256 == 3 || D / 256 == 4 || D / 256 == 8 ||
                       D / 256 == 16)) {
    const int nblk_r = std::min((R + 3) / 4, sms * 4);
    const int rpb = (R + nblk_r - 1) / nblk_r;
    auto part_r = at::empty({nblk_r, D}, x.options().dtype(at::kFloat));
    auto gyp = reinterpret_cast<const __nv_bfloat16*>(gy.data_ptr());
    auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    auto gxp = reinterpret_cast<__nv_bfloat16*>(gx.data_ptr());
    auto launch = [&](auto tag_w, auto nc) {
      using WT = decltype(tag_w);
      constexpr int NC = decltype(nc)::value;
      auto k = rms_bwd_reg_kernel<WT, NC>;
      const int red_bytes = NC * 256 * 4 * (int)sizeof(float);
      if (red_bytes > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, red_bytes);
      k<<<nblk_r, 128, red_bytes, s>>>(gyp, xp, reinterpret_cast<const WT*>(w.data_ptr()), rstd.data_ptr<float>(), gxp,
                               part_r.data_ptr<float>(), R, rpb);
    };
    auto by_nc = [&](auto tag_w) {
      switch (D / 256) {
        case 1: launch(tag_w, std::integral_constant<int, 1>{}); break;
        case 2: launch(tag_w, std::integral_constant<int, 2>{}); break;
        case 3: launch(tag_w, std::integral_constant<int, 3>{}); break;
        case 4: launch(tag_w, std::integral_constant<int, 4>{}); break;
        case 8: launch(tag_w, std::integral_constant<int, 8>{}); break;
        default: launch(tag_w, std::integral_constant<int, 16>{}); break;
      }
    };
    if (w.scalar_type() == at::kFloat)
      by_nc(float{});
    else
      by_nc(__nv_bfloat16{});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    at::sum_out(gw, part_r, 0);
    return;
  }
  const int nblk = std::min((R + warps - 1) / warps, sms * 2);
  const int rows_per_block = (R + nblk - 1) / nblk;
  auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
  auto gyp = reinterpret_cast<const __nv_bfloat16*>(gy.data_ptr());
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto gxp = reinterpret_cast<__nv_bfloat16*>(gx.data_ptr());
  if (w.scalar_type() == at::kFloat) {
    auto k = rms_bwd_kernel<float>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<nblk, warps * 32, smem, s>>>(gyp, xp, w.data_ptr<float>(), rstd.data_ptr<float>(), gxp,
                                     part.data_ptr<float>(), R, D, rows_per_block);
  } else {
    auto k = rms_bwd_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<nblk, warps * 32, smem, s>>>(gyp, xp, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                     rstd.data_ptr<float>(), gxp, part.data_ptr<float>(), R, D, rows_per_block);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  at::sum_out(gw, part, 0);
}

static void check_row_op(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2 && t.is_contiguous() && t.scalar_type() == at::kBFloat16, "dion_b200 ", name,
              ": contiguous [rows, D] bf16 expected");
}

// h = x + a, y = rms_norm(h) * w (D % 256 == 0, 1024 <= D <= 8192)
void add_rms_norm_fwd(const at::Tensor& x, const at::Tensor& a, const at::Tensor& w, at::Tensor& h, at::Tensor& y,
                      at::Tensor& rstd, double eps) {
  check_row_op(x, "add_rms_norm");
  check_row_op(a, "add_rms_norm");
  const int R = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(a.sizes() == x.sizes() && h.sizes() == x.sizes() && y.sizes() == x.sizes() && w.numel() == D &&
                  D % 256 == 0 && D >= 1024 && D <= 8192,
              "dion_b200 add_rms_norm: shapes (D a multiple of 256 in [1024, 8192])");
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = D / 8;
  const int nblk = std::min(R, sms * std::max(1, 2048 / threads));
  const int rpb = (R + nblk - 1) / nblk;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto ap = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  auto hp = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (w.scalar_type() == at::kFloat)
    add_rms_fwd_row_kernel<float><<<nblk, threads, 0, s>>>(xp, ap, w.data_ptr<float>(), hp, yp,
                                                           rstd.data_ptr<float>(), R, D, rpb, (float)eps);
  else
    add_rms_fwd_row_kernel<__nv_bfloat16><<<nblk, threads, 0, s>>>(
        xp, ap, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, yp, rstd.data_ptr<float>(), R, D, rpb,
        (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// gx = gres + d/dh rms_norm(h) . gy ; gw = sum_rows gy * h * rstd
void rms_norm_bwd_res(const at::Tensor& gy, const at::Tensor& h, const at::Tensor& w, const at::Tensor& rstd,
                      const at::Tensor& gres, at::Tensor& gx, at::Tensor& gw) {
  check_row_op(gy, "rms_norm_bwd_res");
  check_row_op(h, "rms_norm_bwd_res");
  check_row_op(gres, "rms_norm_bwd_res");
  const int R = (int)h.size(0), D = (int)h.size(1);
  TORCH_CHECK(D % 256 == 0 && D >= 1024 && D <= 8192 && gres.sizes() == h.sizes() && gy.sizes() == h.sizes(),
              "dion_b200 rms_norm_bwd_res: shapes");
  c10::cuda::CUDAGuard guard(h.device());
  auto s = at::cuda::getCurrentCUDAStream();
  if (R == 0) {
    gw.zero_();
    return;
  }
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = D / 8;
  const int nblk = std::min(R, sms * std::max(1, 2048 / threads));
  const int rpb = (R + nblk - 1) / nblk;
  auto part = at::empty({nblk, D}, h.options().dtype(at::kFloat));
  auto gyp = reinterpret_cast<const __nv_bfloat16*>(gy.data_ptr());
  auto hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  auto rp = reinterpret_cast<const __nv_bfloat16*>(gres.data_ptr());
  auto gxp = reinterpret_cast<__nv_bfloat16*>(gx.data_ptr());
  if (w.scalar_type() == at::kFloat)
    rms_bwd_row_kernel<float><<<nblk, threads, 0, s>>>(gyp, hp, w.data_ptr<float>(), rstd.data_ptr<float>(), gxp,
                                                       part.data_ptr<float>(), R, D, rpb, rp);
  else
    rms_bwd_row_kernel<__nv_bfloat16><<<nblk, threads, 0, s>>>(
        gyp, hp, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(), gxp,
        part.data_ptr<float>(), R, D, rpb, rp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  at::sum_out(gw, part, 0);
}

void rope_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& tab, at::Tensor& qo, at::Tensor& ko,
              bool inverse) {
  TORCH_CHECK(q.dim() == 4 && q.is_contiguous() && k.is_contiguous(), "dion_b200 rope: [b,s,h,d] contiguous");
  c10::cuda::CUDAGuard guard(q.device());
  const int S = (int)q.size(1), hq = (int)q.size(2), hk = (int)k.size(2), d = (int)q.size(3);
  if (d % 8 == 0 && k.size(0) == q.size(0) && k.size(1) == S) {
    const int64_t rows = q.size(0) * (int64_t)S;
    rope_pos_kernel<<<(unsigned)rows, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
        reinterpret_cast<const float2*>(tab.data_ptr<float>()), reinterpret_cast<__nv_bfloat16*>(qo.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(ko.data_ptr()), S, hq, hk, d / 2, inverse ? -1.f : 1.f);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    return;
  }
  if (d % 8 == 0) {
    const int64_t nq8 = q.numel() / 8, nk8 = k.numel() / 8;
    const int64_t grid8 = (nq8 + nk8 + 255) / 256;
    rope8_kernel<<<(unsigned)grid8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
        reinterpret_cast<const float2*>(tab.data_ptr<float>()), reinterpret_cast<__nv_bfloat16*>(qo.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(ko.data_ptr()), nq8, nk8, S, hq, hk, d / 2, inverse ? -1.f : 1.f);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    return;
  }
  const int64_t nq = q.numel() / 2, nk = k.numel() / 2;
  const int threads = 256;
  const int64_t grid = (nq + nk + threads - 1) / threads;
  rope_kernel<<<(unsigned)grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
      tab.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(qo.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(ko.data_ptr()), nq, nk, S, hq, hk, d / 2, inverse ? -1.f : 1.f);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

void swiglu_fwd(const at::Tensor& a, const at::Tensor& b, at::Tensor& o) {
  TORCH_CHECK(a.numel() % 8 == 0, "dion_b200 swiglu: numel % 8");
  c10::cuda::CUDAGuard guard(a.device());
  const int64_t n8 = a.numel() / 8;
  const int grid = (int)std::min<int64_t>((n8 + 255) / 256, 148 * 16);
  swiglu_fwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

void swiglu_bwd(const at::Tensor& g, const at::Tensor& a, const at::Tensor& b, at::Tensor& ga, at::Tensor& gb) {
  c10::cuda::CUDAGuard guard(a.device());
  const int64_t n8 = a.numel() / 8;
  const int grid = (int)std::min<int64_t>((n8 + 255) / 256, 148 * 16);
  swiglu_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()), reinterpret_cast<__nv_bfloat16*>(ga.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(gb.data_ptr()), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

void cross_entropy_fwd_bwd(const at::Tensor& logits, const at::Tensor& labels, at::Tensor& grad, at::Tensor& loss,
                           double scale) {
  TORCH_CHECK(logits.dim() == 2 && logits.is_contiguous() && labels.scalar_type() == at::kLong,
              "dion_b200 cross_entropy: [T, V] bf16 logits, int64 labels");
  TORCH_CHECK(logits.size(1) % 8 == 0, "dion_b200 cross_entropy: V % 8 == 0 required");
  c10::cuda::CUDAGuard guard(logits.device());
  const int T = (int)logits.size(0), V = (int)logits.size(1);
  auto rows = at::empty({T}, logits.options().dtype(at::kFloat));
  ce_kernel<<<T, kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(),
      reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), rows.data_ptr<float>(), V, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  at::sum_out(loss, rows, 0);
}

}  // namespace bdion

// Small dense factorizations for Dion's orthogonalisation (fp32, batched,
// one CTA of 1024 threads per matrix, blocked by 32-column panels):
//
//   cholesky_lower : A = L L^T in place (lower triangle of row-major A)
//   tri_inv_lower  : Z = L^-1 for a lower-triangular L (or L = U^T for an
//                    upper-triangular input), written as a full lower matrix
//   qr_r           : Householder QR of a tall A (m x n, m >= n), R only
//
// Dion needs P R^-1 with R from a QR (randomised sketch) and from a Cholesky
// (CholeskyQR pass); with Z = inv(R^T) lower, P R^-1 = P Z^T, which the
// tcgen05 GEMM reads straight from Z's row-major storage (K-major operand).
//
// Algorithms: right-looking blocked Cholesky (Golub & Van Loan, Alg. 4.2.4
// in blocked form), blocked triangular inversion by row blocks, and blocked
// Householder QR with the compact WY representation (Schreiber & Van Loan
// 1989). Non-positive Cholesky pivots produce NaN (reported per matrix in
// `info`); Dion's all-zero/NaN guard then zeroes the affected update, as the
// reference's cholesky_ex path does.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

namespace {

constexpr int NB = 32;
constexpr int LD = NB + 1;  // padded smem row
constexpr int CT = 1024;
constexpr int QR_CT = 512;  // Householder kernel: two trailing columns per thread, more registers each

__device__ __forceinline__ float block_sum_1024(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32)
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  if (threadIdx.x == 0) red[32] = s;
  __syncthreads();
  return red[32];
}

// ------------------------------------------------------------ Cholesky
__global__ void __launch_bounds__(CT, 1) cholesky_lower_kernel(float* __restrict__ A_all, int r, int64_t bstride,
                                                               int* __restrict__ info) {
  float* A = A_all + (int64_t)blockIdx.x * bstride;
  extern __shared__ float sm[];
  float* sD = sm;            // NB x LD   diagonal block
  float* sP = sm + NB * LD;  // (r) x LD  current panel below the diagonal block
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  for (int k0 = 0; k0 < r; k0 += NB) {
    const int kb = min(NB, r - k0);
    for (int e = threadIdx.x; e < NB * NB; e += CT) {
      const int i = e / NB, j = e % NB;
      sD[i * LD + j] = (i < kb && j <= i) ? A[(int64_t)(k0 + i) * r + k0 + j] : 0.f;
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // unblocked factorization of the diagonal block, lane = row
      const int i = threadIdx.x;
      for (int j = 0; j < kb; ++j) {
        if (i == j) {
          float d = sD[j * LD + j];
          if (!(d > 0.f)) {
            bad = 1;
            d = __int_as_float(0x7fc00000);  // NaN: the caller's guard discards this matrix
          }
          sD[j * LD + j] = sqrtf(d);
        }
        __syncwarp();
        const float djj = sD[j * LD + j];
        if (i > j && i < kb) sD[i * LD + j] /= djj;
        __syncwarp();
        if (i > j && i < kb) {
          const float lij = sD[i * LD + j];
          for (int t = j + 1; t <= i; ++t) sD[i * LD + t] -= lij * sD[t * LD + j];
        }
        __syncwarp();
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kb * kb; e += CT) {
      const int i = e / kb, j = e % kb;
      if (j <= i) A[(int64_t)(k0 + i) * r + k0 + j] = sD[i * LD + j];
    }
    const int rows = r - k0 - kb;
    for (int ii = threadIdx.x; ii < rows; ii += CT) {  // panel: x L_kk^T = a, one row per thread
      const int64_t base = (int64_t)(k0 + kb + ii) * r + k0;
      float x[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) x[j] = j < kb ? A[base + j] : 0.f;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if (j < kb) {
          float s = x[j];
#pragma unroll
          for (int t = 0; t < NB; ++t)
            if (t < j) s -= x[t] * sD[j * LD + t];
          x[j] = s / sD[j * LD + j];
        }
      }
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (j < kb) {
          A[base + j] = x[j];
          sP[ii * LD + j] = x[j];
        }
    }
    __syncthreads();
    // trailing update of the lower triangle, 4x4 tiles per thread
    const int nt = (rows + 3) / 4;
    const int ntiles = nt * (nt + 1) / 2;
    for (int tt = threadIdx.x; tt < ntiles; tt += CT) {
      int ti = (int)((sqrtf(8.f * (float)tt + 1.f) - 1.f) * 0.5f);
      while ((ti + 1) * (ti + 2) / 2 <= tt) ++ti;
      while (ti * (ti + 1) / 2 > tt) --ti;
      const int tj = tt - ti * (ti + 1) / 2;
      float acc[4][4] = {};
      for (int t = 0; t < kb; ++t) {
        float a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ia = ti * 4 + u, jb = tj * 4 + u;
          a[u] = ia < rows ? sP[ia * LD + t] : 0.f;
          b[u] = jb < rows ? sP[jb * LD + t] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) acc[u][v] += a[u] * b[v];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int i = ti * 4 + u, j = tj * 4 + v;
          if (i < rows && j <= i) A[(int64_t)(k0 + kb + i) * r + k0 + kb + j] -= acc[u][v];
        }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && info != nullptr) info[blockIdx.x] = bad;
}

// ------------------------------------------------------------ triangular inverse
// Z = L^-1 (lower). L is the lower triangle of `src` (upper=0) or the
// transpose of its upper triangle (upper=1). Z's strict upper part is zeroed.
__device__ __forceinline__ float tri_get(const float* S, int r, int i, int j, int upper) {
  return upper ? S[(int64_t)j * r + i] : S[(int64_t)i * r + j];
}

__global__ void __launch_bounds__(CT, 1) tri_inv_lower_kernel(const float* __restrict__ S_all, float* __restrict__ Z_all,
                                                              int r, int64_t bstride, int upper) {
  const float* S = S_all + (int64_t)blockIdx.x * bstride;
  float* Z = Z_all + (int64_t)blockIdx.x * bstride;
  extern __shared__ float sm[];
  float* sInv = sm;              // NB x LD  inverse of the diagonal block
  float* sDiag = sm + NB * LD;   // NB x LD  the diagonal block of L
  float* sRow = sm + 2 * NB * LD;  // NB x (r+1) row block of L left of the diagonal
  const int ldr = r + 1;
  for (int64_t e = threadIdx.x; e < (int64_t)r * r; e += CT) {
    const int i = (int)(e / r), j = (int)(e % r);
    if (j > i) Z[e] = 0.f;
  }
  __syncthreads();
  for (int i0 = 0; i0 < r; i0 += NB) {
    const int kb = min(NB, r - i0);
    // diagonal block of L into smem (sDiag), then its inverse by warp 0:
    // lane c solves L_ii x = e_c from shared memory
    for (int e = threadIdx.x; e < NB * NB; e += CT) {
      const int i = e / NB, t = e % NB;
      sDiag[i * LD + t] = (i < kb && t <= i) ? tri_get(S, r, i0 + i, i0 + t, upper) : 0.f;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int c = threadIdx.x;
      float x[NB];
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        float s = (i == c) ? 1.f : 0.f;
#pragma unroll
        for (int t = 0; t < NB; ++t)
          if (t < i) s -= sDiag[i * LD + t] * x[t];
        x[i] = (i < kb && c < kb && i >= c) ? s / sDiag[i * LD + i] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < NB; ++i) sInv[i * LD + c] = x[i];
    }
    // the row block of L left of the diagonal
    for (int e = threadIdx.x; e < kb * i0; e += CT) {
      const int a = e / i0, t = e % i0;
      sRow[a * ldr + t] = tri_get(S, r, i0 + a, t, upper);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kb * kb; e += CT) {
      const int a = e / kb, b = e % kb;
      if (b <= a) Z[(int64_t)(i0 + a) * r + i0 + b] = sInv[a * LD + b];
    }
    // off-diagonal: Z[i-block, c] = -Zii * (L[i-block, 0:i0] Z[0:i0, c]) for c < i0
    for (int c = threadIdx.x; c < i0; c += CT) {
      float s[NB];
#pragma unroll
      for (int a = 0; a < NB; ++a) s[a] = 0.f;
      int t = c;
      for (; t + 8 <= i0; t += 8) {  // 8 independent loads in flight
        float z[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) z[u] = Z[(int64_t)(t + u) * r + c];
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int a = 0; a < NB; ++a) s[a] += sRow[a * ldr + t + u] * z[u];
      }
      for (; t < i0; ++t) {
        const float z = Z[(int64_t)t * r + c];
#pragma unroll
        for (int a = 0; a < NB; ++a) s[a] += sRow[a * ldr + t] * z;
      }
#pragma unroll
      for (int a = 0; a < NB; ++a) {
        if (a < kb) {
          float o = 0.f;
#pragma unroll
          for (int b = 0; b < NB; ++b)
            if (b <= a) o += sInv[a * LD + b] * s[b];
          Z[(int64_t)(i0 + a) * r + c] = -o;
        }
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ Householder QR (R only)
__global__ void __launch_bounds__(QR_CT, 1) qr_r_kernel(float* __restrict__ A_all, int m, int n, int64_t bstride,
                                                     float* __restrict__ R_all, int64_t rstride) {
  float* A = A_all + (int64_t)blockIdx.x * bstride;
  float* R = R_all + (int64_t)blockIdx.x * rstride;
  extern __shared__ float sm[];
  float* sV = sm;                 // rows x LD : the panel, then its Householder vectors
  float* sT = sV + (int64_t)m * LD;  // NB x LD : WY block reflector T
  float* red = sT + NB * LD;      // 40 floats for reductions
  float* sTau = red + 40;         // NB
  float* sBeta = sTau + NB;       // NB
  for (int64_t e = threadIdx.x; e < (int64_t)n * n; e += QR_CT) R[e] = 0.f;
  for (int k0 = 0; k0 < n; k0 += NB) {
    const int kb = min(NB, n - k0);
    const int rows = m - k0;
    for (int64_t e = threadIdx.x; e < (int64_t)rows * NB; e += QR_CT) {
      const int i = (int)(e / NB), j = (int)(e % NB);
      sV[i * LD + j] = j < kb ? A[(int64_t)(k0 + i) * n + k0 + j] : 0.f;
    }
    __syncthreads();
    // unblocked Householder on the panel
    for (int j = 0; j < kb; ++j) {
      float ss = 0.f;
      for (int i = j + 1 + threadIdx.x; i < rows; i += QR_CT) ss += sV[i * LD + j] * sV[i * LD + j];
      const float sigma = block_sum_1024(ss, red);
      const float x0 = sV[j * LD + j];
      float beta, tau, scale;
      if (sigma == 0.f) {
        beta = x0;
        tau = 0.f;
        scale = 0.f;
      } else {
        const float nrm = sqrtf(x0 * x0 + sigma);
        beta = x0 >= 0.f ? -nrm : nrm;
        tau = (beta - x0) / beta;
        scale = 1.f / (x0 - beta);
      }
      for (int i = j + 1 + threadIdx.x; i < rows; i += QR_CT) sV[i * LD + j] *= scale;
      __syncthreads();
      if (threadIdx.x == 0) {
        sTau[j] = tau;
        sBeta[j] = beta;
        sV[j * LD + j] = 1.f;
      }
      __syncthreads();
      // apply (I - tau v v^T) to panel columns j+1..kb-1: one warp per column
      const int w = threadIdx.x / 32, l = threadIdx.x % 32;
      for (int c = j + 1 + w; c < kb; c += QR_CT / 32) {
        float d = 0.f;
        for (int i = j + l; i < rows; i += 32) d += sV[i * LD + j] * sV[i * LD + c];
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffff, d, o);
        const float f = tau * d;
        for (int i = j + l; i < rows; i += 32) sV[i * LD + c] -= f * sV[i * LD + j];
      }
      __syncthreads();
    }
    // R block of this panel (upper part of the factored panel; diagonal = beta)
    for (int e = threadIdx.x; e < kb * kb; e += QR_CT) {
      const int i = e / kb, j = e % kb;
      if (j > i) R[(int64_t)(k0 + i) * n + k0 + j] = sV[i * LD + j];
      if (j == i) R[(int64_t)(k0 + i) * n + k0 + j] = sBeta[i];
    }
    // T of the compact WY form: H_0 ... H_{kb-1} = I - V T V^T
    {
      const int w = threadIdx.x / 32, l = threadIdx.x % 32;
      for (int e = w; e < kb * kb; e += QR_CT / 32) {  // dots V[:,a]^T V[:,b], a < b
        const int a = e / kb, b = e % kb;
        if (a < b) {
          float d = 0.f;
          for (int i = b + l; i < rows; i += 32) {
            const float va = (i == a) ? 1.f : (i > a ? sV[i * LD + a] : 0.f);
            d += va * sV[i * LD + b];
          }
          for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffff, d, o);
          if (l == 0) sT[a * LD + b] = d;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {  // T[:, j] = -tau_j T[:, :j] (V^T v_j)
        float tmp[NB];
        for (int j = 0; j < kb; ++j) {
          for (int a = 0; a < j; ++a) tmp[a] = sT[a * LD + j];
          for (int a = 0; a < j; ++a) {
            float s = 0.f;
            for (int b = a; b < j; ++b) s += sT[a * LD + b] * tmp[b];
            sT[a * LD + j] = -sTau[j] * s;
          }
          sT[j * LD + j] = sTau[j];
          for (int a = j + 1; a < NB; ++a) sT[a * LD + j] = 0.f;
        }
      }
      __syncthreads();
    }
    // trailing columns: C -= V (T^T (V^T C)), one column per thread
    const int nc = n - k0 - kb;
    for (int c = threadIdx.x; c < nc; c += QR_CT) {
      const int col = k0 + kb + c;
      float wv[NB];
#pragma unroll
      for (int a = 0; a < NB; ++a) wv[a] = 0.f;
      float* Ac = A + (int64_t)k0 * n + col;
      const int ktri = min(kb, rows);
      // rows inside the triangular head of V (unit diagonal, zeros above)
      for (int i = 0; i < ktri; ++i) {
        const float cv = Ac[(int64_t)i * n];
#pragma unroll
        for (int a = 0; a < NB; ++a) {
          const float va = (i == a) ? 1.f : (i > a ? sV[i * LD + a] : 0.f);
          wv[a] += va * cv;
        }
      }
      // dense rows: 8 independent loads in flight per step
      int i = ktri;
      for (; i + 8 <= rows; i += 8) {
        float cv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) cv[u] = Ac[(int64_t)(i + u) * n];
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int a = 0; a < NB; ++a) wv[a] += sV[(i + u) * LD + a] * cv[u];
      }
      for (; i < rows; ++i) {
        const float cv = Ac[(int64_t)i * n];
#pragma unroll
        for (int a = 0; a < NB; ++a) wv[a] += sV[i * LD + a] * cv;
      }
      // wv <- T^T wv in place (row a only needs entries b <= a, so go downwards)
#pragma unroll
      for (int a = NB - 1; a >= 0; --a) {
        float sacc = 0.f;
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b <= a) sacc += sT[b * LD + a] * wv[b];
        wv[a] = a < kb ? sacc : 0.f;
      }
      float* Rc = R + (int64_t)k0 * n + col;
      for (int i2 = 0; i2 < ktri; ++i2) {
        float sacc = 0.f;
#pragma unroll
        for (int a = 0; a < NB; ++a) {
          const float va = (i2 == a) ? 1.f : (i2 > a ? sV[i2 * LD + a] : 0.f);
          sacc += va * wv[a];
        }
        const float nv = Ac[(int64_t)i2 * n] - sacc;
        Ac[(int64_t)i2 * n] = nv;
        Rc[(int64_t)i2 * n] = nv;
      }
      i = ktri;
      for (; i + 8 <= rows; i += 8) {
        float sv8[8], cv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) cv[u] = Ac[(int64_t)(i + u) * n];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float sacc = 0.f;
#pragma unroll
          for (int a = 0; a < NB; ++a) sacc += sV[(i + u) * LD + a] * wv[a];
          sv8[u] = sacc;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) Ac[(int64_t)(i + u) * n] = cv[u] - sv8[u];
      }
      for (; i < rows; ++i) {
        float sacc = 0.f;
#pragma unroll
        for (int a = 0; a < NB; ++a) sacc += sV[i * LD + a] * wv[a];
        Ac[(int64_t)i * n] -= sacc;
      }
    }
    __syncthreads();
  }
}

}  // namespace

// A: [b, r, r] fp32 contiguous, overwritten with L in its lower triangle.
void cholesky_lower(at::Tensor& A, at::Tensor& info) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) == A.size(2),
              "dion_b200 cholesky: contiguous [b, r, r] fp32");
  const int b = (int)A.size(0), r = (int)A.size(1);
  const size_t smem = (size_t)(NB * LD + (size_t)r * LD) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "dion_b200 cholesky: r too large for the single-CTA kernel");
  c10::cuda::CUDAGuard guard(A.device());
  cudaFuncSetAttribute(cholesky_lower_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cholesky_lower_kernel<<<b, CT, smem, at::cuda::getCurrentCUDAStream()>>>(A.data_ptr<float>(), r, (int64_t)r * r,
                                                                            info.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// S: [b, r, r] fp32 (lower, or upper if `upper`); Z: [b, r, r] = inv(L) lower.
void tri_inv_lower(const at::Tensor& S, at::Tensor& Z, bool upper) {
  TORCH_CHECK(S.dim() == 3 && S.is_contiguous() && Z.is_contiguous() && S.scalar_type() == at::kFloat,
              "dion_b200 tri_inv: contiguous [b, r, r] fp32");
  const int b = (int)S.size(0), r = (int)S.size(1);
  const size_t smem = (size_t)(2 * NB * LD + (size_t)NB * (r + 1)) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "dion_b200 tri_inv: r too large");
  c10::cuda::CUDAGuard guard(S.device());
  cudaFuncSetAttribute(tri_inv_lower_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  tri_inv_lower_kernel<<<b, CT, smem, at::cuda::getCurrentCUDAStream()>>>(S.data_ptr<float>(), Z.data_ptr<float>(),
                                                                           r, (int64_t)r * r, upper ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// A: [b, m, n] fp32 contiguous (m >= n), overwritten; R: [b, n, n] upper.
void qr_r(at::Tensor& A, at::Tensor& R) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) >= A.size(2),
              "dion_b200 qr_r: contiguous [b, m, n] fp32 with m >= n");
  const int b = (int)A.size(0), m = (int)A.size(1), n = (int)A.size(2);
  const size_t smem = ((size_t)m * LD + NB * LD + 40 + 2 * NB) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "dion_b200 qr_r: m too large for the single-CTA kernel");
  c10::cuda::CUDAGuard guard(A.device());
  cudaFuncSetAttribute(qr_r_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  qr_r_kernel<<<b, QR_CT, smem, at::cuda::getCurrentCUDAStream()>>>(A.data_ptr<float>(), m, n, (int64_t)m * n,
                                                                  R.data_ptr<float>(), (int64_t)n * n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace bdion

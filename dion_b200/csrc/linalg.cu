// Small dense factorizations for Dion's orthogonalisation (fp32, batched,
// blocked by 32-column panels; each matrix is handled by a thread-block
// cluster of up to 8 CTAs sized so the batch covers the SMs -- the panel
// work is repeated in every CTA of the cluster, the trailing update is split
// across them, and a hardware cluster barrier separates block steps):
//
//   cholesky_lower : A = L L^T in place (lower triangle of row-major A)
//   tri_inv_lower  : Z = L^-1 for a lower-triangular L (or L = U^T for an
//                    upper-triangular input), written as a full lower matrix
//                    (recursive doubling over batched fp32 GEMMs, below)
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
constexpr int QR_CT = 256;  // Householder kernel: 32 accumulators per trailing column, no register spills

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
// Barrier over every thread of every CTA of this thread-block cluster, with
// release/acquire ordering of global-memory accesses at cluster scope (a
// hardware barrier: no memory polling).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Cluster of `nclus` CTAs per matrix: every CTA factors the diagonal block
// and solves the panel itself (cheap, and it keeps panel data local), the
// trailing-triangle tiles are split over the CTAs, and a cluster barrier
// orders each block step's updates before the next step reads them.
__global__ void __launch_bounds__(CT, 1) cholesky_lower_kernel(float* __restrict__ A_all, int r, int64_t bstride,
                                                               int* __restrict__ info, int nclus) {
  const int crank = (int)(blockIdx.x % nclus);
  const int mat = (int)(blockIdx.x / nclus);
  float* A = A_all + (int64_t)mat * bstride;
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
        if (j < kb) sP[ii * LD + j] = x[j];
    }
    __syncthreads();
    // trailing update of the lower triangle, 4x4 tiles per thread, tiles split over the cluster
    const int nt = (rows + 3) / 4;
    const int ntiles = nt * (nt + 1) / 2;
    for (int tt = crank * CT + threadIdx.x; tt < ntiles; tt += nclus * CT) {
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
    cluster_sync_all();
    // the factored block column goes back to A only now: every CTA has read
    // this step's inputs, and later steps never read these columns
    if (crank == 0) {
      for (int e = threadIdx.x; e < kb * kb; e += CT) {
        const int i = e / kb, j = e % kb;
        if (j <= i) A[(int64_t)(k0 + i) * r + k0 + j] = sD[i * LD + j];
      }
      for (int64_t e = threadIdx.x; e < (int64_t)rows * kb; e += CT) {
        const int ii = (int)(e / kb), j = (int)(e % kb);
        A[(int64_t)(k0 + kb + ii) * r + k0 + j] = sP[ii * LD + j];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && crank == 0 && info != nullptr) info[mat] = bad;
}

// ------------------------------------------------------------ triangular inverse
// Z = L^-1 (lower). L is the lower triangle of `src` (upper=0) or the
// transpose of its upper triangle (upper=1). Z's strict upper part is zeroed.
__device__ __forceinline__ float tri_get(const float* S, int r, int i, int j, int upper) {
  return upper ? S[(int64_t)j * r + i] : S[(int64_t)i * r + j];
}

// ------------------------------------------------------------ triangular inverse by recursive doubling
// L^-1 for lower-triangular L, level by level: all 32x32 diagonal blocks are
// inverted independently, then blocks of size s are paired into 2s:
//     [L11  0 ]^-1   [ Z11          0  ]
//     [L21 L22]    = [ -Z22 L21 Z11  Z22 ],   Z21 = -Z22 (L21 Z11)
// which is two batched fp32 GEMMs per level (log2(r/32) levels), every
// pair of every matrix in parallel across the GPU.

// one warp per 32x32 diagonal block: lane c solves L_jj x = e_c (forward substitution)
__global__ void tri_inv_diag_kernel(const float* __restrict__ S_all, float* __restrict__ Z_all, int r,
                                    int64_t bstride, int upper) {
  const int mat = blockIdx.y;
  const int blk = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int c = threadIdx.x % 32;
  const int nblk = (r + NB - 1) / NB;
  if (blk >= nblk) return;
  const float* S = S_all + (int64_t)mat * bstride;
  float* Z = Z_all + (int64_t)mat * bstride;
  const int i0 = blk * NB, kb = min(NB, r - i0);
  __shared__ float sD[4][NB][LD];
  float (*D)[LD] = sD[threadIdx.x / 32];
  for (int i = 0; i < NB; ++i) D[i][c] = (i < kb && c <= i) ? tri_get(S, r, i0 + i, i0 + c, upper) : 0.f;
  __syncwarp();
  float x[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    float s2 = (i == c) ? 1.f : 0.f;
#pragma unroll
    for (int t = 0; t < NB; ++t)
      if (t < i) s2 -= D[i][t] * x[t];
    x[i] = (i < kb && c < kb && i >= c) ? s2 / D[i][i] : 0.f;
  }
  // row i0+i of Z: x[i] in column i0+c; zero the rest of the row band above the diagonal
  if (c < kb) {
#pragma unroll
    for (int i = 0; i < NB; ++i)
      if (i < kb) Z[(int64_t)(i0 + i) * r + i0 + c] = x[i];
  }
  for (int i = 0; i < kb; ++i)
    for (int j = i0 + NB + c; j < r; j += 32) Z[(int64_t)(i0 + i) * r + j] = 0.f;
}

// C[z] = alpha * A[z] @ B[z] (M x K @ K x N), fp32 FMA, 64x64 tiles, 4x4 per thread.
// Operand z = (matrix b, pair p): base + b*bstride + p*pstride + off, element
// (i, j) at i*rs + j*cs (any strides: covers transposed views).
struct Opnd {
  const float* base;
  int64_t bstride, pstride, off, rs, cs;
  __device__ __forceinline__ const float* at(int b, int p) const { return base + b * bstride + p * pstride + off; }
};

__global__ void __launch_bounds__(256) sgemm_pairs_kernel(Opnd A, Opnd B, float* Cbase, int64_t c_bstride,
                                                          int64_t c_pstride, int64_t c_off, int64_t c_rs, int M,
                                                          int N, int K, int pairs, float alpha) {
  const int z = blockIdx.z;
  const int b = z / pairs, p = z % pairs;
  const float* Ap = A.at(b, p);
  const float* Bp = B.at(b, p);
  float* Cp = Cbase + b * c_bstride + p * c_pstride + c_off;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      const int kk = e / 64, mm = e % 64;
      const int gi = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gi < M && gk < K) ? Ap[gi * A.rs + gk * A.cs] : 0.f;
      const int gn = n0 + mm;
      Bs[kk][mm] = (gk < K && gn < N) ? Bp[gk * B.rs + gn * B.cs] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = As[kk][ty * 4 + u];
        bb[u] = Bs[kk][tx * 4 + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] += a[u] * bb[v];
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int gi = m0 + ty * 4 + u, gj = n0 + tx * 4 + v;
      if (gi < M && gj < N) Cp[gi * c_rs + gj] = alpha * acc[u][v];
    }
}

// ------------------------------------------------------------ Householder QR (R only)
// One thread-block cluster of `nclus` CTAs per matrix (cluster dims set at
// launch). Every CTA factors the current 32-column panel itself (read from
// global memory, so no panel data crosses CTAs) and applies the block
// reflector to the trailing column blocks it owns (block jb belongs to CTA
// jb % nclus); a cluster barrier (release/acquire) after each panel makes
// the owners' updated columns visible before the next panel is read. With
// nclus = 1 this is the single-CTA algorithm.
constexpr int QLD = NB + 4;  // panel row stride: 16-byte rows for vector reads of V

__global__ void __launch_bounds__(QR_CT, 1) qr_r_kernel(float* __restrict__ A_all, int m, int n, int64_t bstride,
                                                     float* __restrict__ R_all, int64_t rstride, int nclus) {
  const int crank = (int)(blockIdx.x % nclus);
  const int mat = (int)(blockIdx.x / nclus);
  float* A = A_all + (int64_t)mat * bstride;
  float* R = R_all + (int64_t)mat * rstride;
  extern __shared__ __align__(16) float sm[];
  float* sV = sm;                     // rows x QLD : the panel, then its Householder vectors
  float* sT = sV + (int64_t)m * QLD;  // NB x LD : WY block reflector T
  float* red = sT + NB * LD;          // 40 floats for reductions
  float* sTau = red + 40;             // NB
  float* sBeta = sTau + NB;           // NB
  // strictly-lower part of R is zero; everything else is written by the panel
  // loop (no overlap, so no ordering with the other CTAs is needed)
  for (int64_t e = (int64_t)crank * QR_CT + threadIdx.x; e < (int64_t)n * n; e += (int64_t)nclus * QR_CT)
    if (e % n < e / n) R[e] = 0.f;
  const int nblk = (n + NB - 1) / NB;
  for (int k0 = 0; k0 < n; k0 += NB) {
    const int kb = min(NB, n - k0);
    const int rows = m - k0;
    for (int64_t e = threadIdx.x; e < (int64_t)rows * NB; e += QR_CT) {
      const int i = (int)(e / NB), j = (int)(e % NB);
      sV[i * QLD + j] = j < kb ? A[(int64_t)(k0 + i) * n + k0 + j] : 0.f;
    }
    __syncthreads();
    // unblocked Householder on the panel
    for (int j = 0; j < kb; ++j) {
      float ss = 0.f;
      for (int i = j + 1 + threadIdx.x; i < rows; i += QR_CT) ss += sV[i * QLD + j] * sV[i * QLD + j];
      const float sigma = block_sum_1024(ss, red);
      const float x0 = sV[j * QLD + j];
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
      for (int i = j + 1 + threadIdx.x; i < rows; i += QR_CT) sV[i * QLD + j] *= scale;
      __syncthreads();
      if (threadIdx.x == 0) {
        sTau[j] = tau;
        sBeta[j] = beta;
        sV[j * QLD + j] = 1.f;
      }
      __syncthreads();
      // apply (I - tau v v^T) to panel columns j+1..kb-1: one warp per column
      const int w = threadIdx.x / 32, l = threadIdx.x % 32;
      for (int c = j + 1 + w; c < kb; c += QR_CT / 32) {
        float d = 0.f;
        for (int i = j + l; i < rows; i += 32) d += sV[i * QLD + j] * sV[i * QLD + c];
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffff, d, o);
        const float f = tau * d;
        for (int i = j + l; i < rows; i += 32) sV[i * QLD + c] -= f * sV[i * QLD + j];
      }
      __syncthreads();
    }
    // R block of this panel (upper part of the factored panel; diagonal = beta): panel owner only
    if ((k0 / NB) % nclus == crank) {
      for (int e = threadIdx.x; e < kb * kb; e += QR_CT) {
        const int i = e / kb, j = e % kb;
        if (j > i) R[(int64_t)(k0 + i) * n + k0 + j] = sV[i * QLD + j];
        if (j == i) R[(int64_t)(k0 + i) * n + k0 + j] = sBeta[i];
      }
    }
    // T of the compact WY form: H_0 ... H_{kb-1} = I - V T V^T
    {
      const int w = threadIdx.x / 32, l = threadIdx.x % 32;
      for (int e = w; e < kb * kb; e += QR_CT / 32) {  // dots V[:,a]^T V[:,b], a < b
        const int a = e / kb, b = e % kb;
        if (a < b) {
          float d = 0.f;
          for (int i = b + l; i < rows; i += 32) {
            const float va = (i == a) ? 1.f : (i > a ? sV[i * QLD + a] : 0.f);
            d += va * sV[i * QLD + b];
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
            float s2 = 0.f;
            for (int b = a; b < j; ++b) s2 += sT[a * LD + b] * tmp[b];
            sT[a * LD + j] = -sTau[j] * s2;
          }
          sT[j * LD + j] = sTau[j];
          for (int a = j + 1; a < NB; ++a) sT[a * LD + j] = 0.f;
        }
      }
      __syncthreads();
    }
    // trailing columns this CTA owns: C -= V (T^T (V^T C)). `spl` consecutive
    // lanes share a column when the CTA owns fewer columns than threads: each
    // takes the rows i % spl == part, the partial V^T C are summed with warp
    // shuffles, and each lane updates its own rows.
    const int jb0 = k0 / NB + 1;
    const int jfirst = jb0 + ((crank - jb0 % nclus) % nclus + nclus) % nclus;
    const int owned = jfirst < nblk ? (nblk - 1 - jfirst) / nclus + 1 : 0;
    const int owned_cols = owned * NB;
    int spl = 1;
    while (spl < 8 && owned_cols * spl * 2 <= QR_CT) spl *= 2;
    for (int t = threadIdx.x; t < owned_cols * spl; t += QR_CT) {
      const int ci = t / spl, part = t % spl;
      const int col = (jfirst + (ci / NB) * nclus) * NB + ci % NB;
      if (col >= n) continue;
      float wv[NB];
#pragma unroll
      for (int a = 0; a < NB; ++a) wv[a] = 0.f;
      float* Ac = A + (int64_t)k0 * n + col;
      const int ktri = min(kb, rows);
      const int d0 = ktri + ((part - ktri % spl) % spl + spl) % spl;  // first dense row of this lane
      // rows inside the triangular head of V (unit diagonal, zeros above)
      for (int i = part; i < ktri; i += spl) {
        const float cv = Ac[(int64_t)i * n];
#pragma unroll
        for (int a = 0; a < NB; ++a) {
          const float va = (i == a) ? 1.f : (i > a ? sV[i * QLD + a] : 0.f);
          wv[a] += va * cv;
        }
      }
      // dense rows: 8 independent loads in flight, V rows read as float4 broadcasts
      int i = d0;
      for (; i + 7 * spl < rows; i += 8 * spl) {
        float cv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) cv[u] = Ac[(int64_t)(i + u * spl) * n];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4* vr = reinterpret_cast<const float4*>(sV + (i + u * spl) * QLD);
#pragma unroll
          for (int a4 = 0; a4 < NB / 4; ++a4) {
            const float4 v4 = vr[a4];
            wv[4 * a4 + 0] += v4.x * cv[u];
            wv[4 * a4 + 1] += v4.y * cv[u];
            wv[4 * a4 + 2] += v4.z * cv[u];
            wv[4 * a4 + 3] += v4.w * cv[u];
          }
        }
      }
      for (; i < rows; i += spl) {
        const float cv = Ac[(int64_t)i * n];
#pragma unroll
        for (int a = 0; a < NB; ++a) wv[a] += sV[i * QLD + a] * cv;
      }
      if (spl > 1) {  // the lanes of one column are consecutive in a warp and active together
        const unsigned mask = __activemask();
        for (int o = 1; o < spl; o <<= 1)
#pragma unroll
          for (int a = 0; a < NB; ++a) wv[a] += __shfl_xor_sync(mask, wv[a], o);
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
      for (int i2 = part; i2 < ktri; i2 += spl) {
        float sacc = 0.f;
#pragma unroll
        for (int a = 0; a < NB; ++a) {
          const float va = (i2 == a) ? 1.f : (i2 > a ? sV[i2 * QLD + a] : 0.f);
          sacc += va * wv[a];
        }
        const float nv = Ac[(int64_t)i2 * n] - sacc;
        Ac[(int64_t)i2 * n] = nv;
        Rc[(int64_t)i2 * n] = nv;
      }
      i = d0;
      for (; i + 7 * spl < rows; i += 8 * spl) {
        float sv8[8], cv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) cv[u] = Ac[(int64_t)(i + u * spl) * n];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4* vr = reinterpret_cast<const float4*>(sV + (i + u * spl) * QLD);
          float sacc = 0.f;
#pragma unroll
          for (int a4 = 0; a4 < NB / 4; ++a4) {
            const float4 v4 = vr[a4];
            sacc += v4.x * wv[4 * a4] + v4.y * wv[4 * a4 + 1] + v4.z * wv[4 * a4 + 2] + v4.w * wv[4 * a4 + 3];
          }
          sv8[u] = sacc;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) Ac[(int64_t)(i + u * spl) * n] = cv[u] - sv8[u];
      }
      for (; i < rows; i += spl) {
        float sacc = 0.f;
#pragma unroll
        for (int a = 0; a < NB; ++a) sacc += sV[i * QLD + a] * wv[a];
        Ac[(int64_t)i * n] -= sacc;
      }
    }
    // owners' updated columns -> visible to every CTA of the cluster before the next panel
    cluster_sync_all();
  }
}

}  // namespace

// CTAs per matrix for the clustered kernels: enough to cover the SMs, at
// most 8 (the portable cluster size; 16-CTA clusters measured 2x slower for
// a batch of 8: fewer of them are co-resident), 1 when the batch alone fills
// the GPU.
template <typename Kern, typename... Args>
void launch_clustered(Kern kern, int batch, int threads, size_t smem, Args... args) {
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nclus = 1;
  while (nclus < 8 && batch * nclus * 2 <= sms) nclus *= 2;
  cfg.gridDim = dim3((unsigned)(batch * nclus));
  attr[0].val.clusterDim.x = (unsigned)nclus;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, args..., nclus));
  note_launch();
}

// A: [b, r, r] fp32 contiguous, overwritten with L in its lower triangle.
void cholesky_lower(at::Tensor& A, at::Tensor& info) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) == A.size(2),
              "dion_b200 cholesky: contiguous [b, r, r] fp32");
  const int b = (int)A.size(0), r = (int)A.size(1);
  if (b == 0 || A.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  const size_t smem = (size_t)(NB * LD + (size_t)r * LD) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "dion_b200 cholesky: r too large for the single-CTA kernel");
  c10::cuda::CUDAGuard guard(A.device());
  launch_clustered(cholesky_lower_kernel, b, CT, smem, A.data_ptr<float>(), r, (int64_t)r * r,
                   info.data_ptr<int>());
}

// S: [b, r, r] fp32 (lower, or upper if `upper`); Z: [b, r, r] = inv(L) lower.
void tri_inv_lower(const at::Tensor& S, at::Tensor& Z, bool upper) {
  TORCH_CHECK(S.dim() == 3 && S.is_contiguous() && Z.is_contiguous() && S.scalar_type() == at::kFloat,
              "dion_b200 tri_inv: contiguous [b, r, r] fp32");
  const int b = (int)S.size(0), r = (int)S.size(1);
  if (b == 0 || S.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  c10::cuda::CUDAGuard guard(S.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int nblk = (r + NB - 1) / NB;
  const int64_t bs = (int64_t)r * r;
  tri_inv_diag_kernel<<<dim3((unsigned)((nblk + 3) / 4), (unsigned)b), 128, 0, stream>>>(
      S.data_ptr<float>(), Z.data_ptr<float>(), r, bs, upper ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
  // scratch for T = L21 Z11 of every pair of every matrix at the current level
  // (per level: pairs x s2 x s <= r x r per matrix)
  at::Tensor T = at::empty({(int64_t)b * r * r}, S.options());
  const float* Sp = S.data_ptr<float>();
  float* Zp = Z.data_ptr<float>();
  for (int s = NB; s < r; s *= 2) {
    const int pairs = (r - s + 2 * s - 1) / (2 * s);  // pairs whose L22 block exists (may be partial)
    // partial last pair: L22 rows [2ks+s, min(r, 2ks+2s)); sizes differ only for the last pair,
    // so launch full pairs and the ragged last pair separately
    const int full = (r / (2 * s));
    for (int part = 0; part < 2; ++part) {
      const int np = part == 0 ? full : pairs - full;
      if (np <= 0) continue;
      const int p0 = part == 0 ? 0 : full;
      const int s2 = part == 0 ? s : r - (p0 * 2 * s + s);  // rows of L22 / Z22
      const int64_t pstr = (int64_t)2 * s * r + 2 * s;       // next pair: 2s rows and 2s columns on
      const int64_t o0 = (int64_t)p0 * pstr;
      // L21 (s2 x s): rows 2ks+s.., columns 2ks..; for an upper input L = S^T
      Opnd L21{Sp, bs, pstr, 0, 0, 0};
      if (!upper) {
        L21.off = o0 + (int64_t)s * r;
        L21.rs = r;
        L21.cs = 1;
      } else {
        L21.off = o0 + s;
        L21.rs = 1;
        L21.cs = r;
      }
      Opnd Z11{Zp, bs, pstr, o0, r, 1};
      float* Tp = T.data_ptr<float>();
      const int64_t t_pstr = (int64_t)s2 * s;
      dim3 g1((unsigned)((s + 63) / 64), (unsigned)((s2 + 63) / 64), (unsigned)(b * np));
      sgemm_pairs_kernel<<<g1, 256, 0, stream>>>(L21, Z11, Tp, (int64_t)np * t_pstr, t_pstr, 0, s, s2, s, s, np,
                                                 1.f);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      note_launch();
      Opnd Z22{Zp, bs, pstr, o0 + (int64_t)s * r + s, r, 1};
      Opnd Tm{Tp, (int64_t)np * t_pstr, t_pstr, 0, s, 1};
      sgemm_pairs_kernel<<<g1, 256, 0, stream>>>(Z22, Tm, Zp, bs, pstr, o0 + (int64_t)s * r, r, s2, s, s2, np,
                                                 -1.f);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      note_launch();
    }
  }
}

// A: [b, m, n] fp32 contiguous (m >= n), overwritten; R: [b, n, n] upper.
// Cluster size: enough CTAs per matrix to cover the SMs (at most 8, the
// portable cluster size), 1 when the batch alone fills the GPU.
void qr_r(at::Tensor& A, at::Tensor& R) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) >= A.size(2),
              "dion_b200 qr_r: contiguous [b, m, n] fp32 with m >= n");
  const int b = (int)A.size(0), m = (int)A.size(1), n = (int)A.size(2);
  if (b == 0 || A.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  const size_t smem = ((size_t)m * QLD + NB * LD + 40 + 2 * NB) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "dion_b200 qr_r: m too large for the panel kernel");
  c10::cuda::CUDAGuard guard(A.device());
  launch_clustered(qr_r_kernel, b, QR_CT, smem, A.data_ptr<float>(), m, n, (int64_t)m * n, R.data_ptr<float>(),
                   (int64_t)n * n);
}

}  // namespace bdion

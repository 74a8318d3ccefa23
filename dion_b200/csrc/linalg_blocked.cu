// Blocked Householder QR (R only) and blocked Cholesky whose trailing updates
// run on the tcgen05 tensor cores (batched, fp32 in / fp32 out).
//
// Both factorizations step over 32-column panels. The column-sequential work
// of a panel runs in one kernel on CUDA cores in fp32; the bulk of the flops
// (the trailing update) is a tensor-core GEMM of the package's tcgen05 kernel.
// That GEMM reads fp32 operands as tf32 (10-bit mantissa), so the rank-32
// products are evaluated as three tf32 products (Markidis et al. 2018,
// "3xTF32"): x = hi(x) + lo(x) with hi = round-to-tf32(x), and
//     X Y ~ Xhi Yhi + Xhi Ylo + Xlo Yhi,
// which one GEMM computes when the operands are concatenated along K
// ([Xhi | Xhi | Xlo] times [Yhi ; Ylo ; Yhi], K = 96). The panel kernels write
// their factors in that split form, so the update has fp32-level accuracy
// (the sketch QR of Dion's randomised Cholesky QR must stay stable for
// ill-conditioned P, which plain tf32 updates would not give).
//
// QR (compact WY, Schreiber & Van Loan 1989), per 32-column panel j0:
//   1. qr_panel_kernel : Householder vectors of A[j0:, j0:j0+32] (in place,
//      R block written), V (explicit, unit diagonal; fp32 and split) and the
//      upper-triangular T (32 x 32) of H_0 ... H_31 = I - V T V^T;
//   2. qr_w_kernel     : W' = T^T (V^T A[j0:, j0+32:]) (fp32, CUDA cores),
//      written split as [W'hi ; W'lo ; W'hi];
//   3. tcgen05 GEMM    : A[j0:, j0+32:] -= V W'  (in place, 3xTF32).
//   Q^T = I - V T^T V^T, so step 3 applies Q^T of the panel to the trailing
//   columns. R is the upper triangle of A[:n, :n] at the end.
// Cholesky (right-looking, Golub & Van Loan Alg. 4.2.4 in blocked form):
//   1. chol_panel_kernel : L11 = chol(A11) (one warp) and L21 = A21 L11^-T
//      (one thread per row), written into A and, split, into two K = 96
//      operand buffers;
//   2. tcgen05 GEMM (symmetric mode) : A22 -= L21 L21^T in place.
// A non-positive pivot gives NaN and info[mat] = 1 (as cholesky_ex reports).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "host_utils.h"

namespace bdion {

void gemm_ex(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& C,
             double alpha, double beta, const c10::optional<at::Tensor>& scale, int64_t alpha_pow, int64_t beta_pow,
             bool sym, bool param_mode, double gamma, double delta, int64_t bn_pref,
             const c10::optional<at::Tensor>& D_ptrs, int64_t ldd_ptrs, int64_t out_dtype_ptrs, int64_t nrep,
             int64_t rows_per_ptr, int64_t rot_b, int64_t rot_rows);

namespace {

constexpr int PB = 32;        // panel width
constexpr int PLD = PB + 1;   // padded shared-memory row
constexpr int KC = 3 * PB;    // K of the split (3xTF32) rank-32 update
constexpr int QP_T = 1024;    // QR panel kernel: 32 warps, lane = panel column
constexpr int QP_W = QP_T / 32;
constexpr int kQrMaxChunk = 1400;  // panel rows one CTA can keep in shared memory
constexpr int kQrDefaultChunk = 640;  // default rows per CTA (measured: 640 ~ 1400 > 320 > 160)

__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Barrier over the CTA (nclus == 1) or over every thread of the cluster, with
// release/acquire ordering of shared-memory writes at cluster scope.
__device__ __forceinline__ void panel_sync(int nclus) {
  if (nclus == 1) {
    __syncthreads();
  } else {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
}

__device__ __forceinline__ float ld_cluster_f32(const float* local_addr, int cta) {
  uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(local_addr));
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(sa), "r"(cta));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// ------------------------------------------------------------ QR panel
// One matrix per cluster of `nclus` CTAs (nclus = 1: one CTA). CTA q holds
// panel rows [q*chunk, min(rows, (q+1)*chunk)) in shared memory; the first
// 32 rows (the R block) are always in CTA 0. Thread (warp w, lane c) owns
// column c of the local rows w, w + 32, ... . A column step j takes two
// reductions over rows, each closed by one barrier:
//   (a) sigma = sum of squares of column j below the diagonal (accumulated
//       by lane j during the previous step's update);
//   (b) D_c = sum_{i>j} a_ij a_ic for every column c. For c > j this gives
//       v_j^T a_c for the update; for c < j, where column c already holds
//       v_c, it gives v_c^T v_j, the entries of V^T V that T needs -- so the
//       compact-WY factor costs no extra pass over the panel.
// The update a_ic -= coef_c a_ij (coef_j = 1 - scale turns column j into v_j)
// also accumulates the next column's sum of squares.
__global__ void __launch_bounds__(QP_T, 1)
    qr_panel_kernel(float* __restrict__ A_all, int m, int n, int64_t bstride, int j0, int kb, int chunk,
                    float* __restrict__ Vg_all, float* __restrict__ Vc_all, float* __restrict__ Tg_all,
                    int64_t vstride, int64_t cstride, int nclus) {
  const int crank = (int)(blockIdx.x % nclus);
  const int mat = (int)(blockIdx.x / nclus);
  const int rows = m - j0;
  const int r0 = crank * chunk;
  const int nloc = max(0, min(chunk, rows - r0));
  float* A = A_all + (int64_t)mat * bstride + (int64_t)j0 * n + j0;  // panel origin, row stride n
  float* Vg = Vg_all + (int64_t)mat * vstride;
  float* Vc = Vc_all + (int64_t)mat * cstride;
  float* Tg = Tg_all + (int64_t)mat * PB * PB;

  extern __shared__ __align__(16) float sm[];
  float* sA = sm;                             // chunk x PLD
  float* red_ss = sA + (int64_t)chunk * PLD;  // QP_W
  float* red_dot = red_ss + QP_W;             // QP_W x PLD
  float* cta_vec = red_dot + QP_W * PLD;      // 2 + PB : [sum of squares, x0, row j]  (cluster mode)
  float* cta_dot = cta_vec + 2 + PB;          // PB                                    (cluster mode)
  float* sG = cta_dot + PB;                   // PB x PLD : G[b][j] = v_b^T v_j (b < j)
  float* sTau = sG + PB * PLD;                // PB
  float* sBeta = sTau + PB;                   // PB

  const int w = threadIdx.x / 32, c = threadIdx.x % 32;
  for (int e = threadIdx.x; e < nloc * PB; e += QP_T) {
    const int i = e / PB, cc = e % PB;
    sA[i * PLD + cc] = cc < kb ? A[(int64_t)(r0 + i) * n + cc] : 0.f;
  }
  __syncthreads();
  // sum of squares of this thread's rows below row 0 (lane 0's value starts step 0)
  float ss = 0.f;
  for (int li = w; li < nloc; li += QP_W)
    if (r0 + li > 0) {
      const float x = sA[li * PLD + c];
      ss += x * x;
    }

  for (int j = 0; j < kb; ++j) {
    // ---- (a) sigma and x0
    if (c == j) red_ss[w] = ss;
    __syncthreads();
    float sigma = 0.f;
#pragma unroll 8
    for (int q = 0; q < QP_W; ++q) sigma += red_ss[q];
    float x0, ajc;
    if (nclus == 1) {
      x0 = sA[j * PLD + j];
      ajc = sA[j * PLD + c];
    } else {
      if (threadIdx.x == 0) cta_vec[0] = sigma;
      if (crank == 0 && w == 0) {
        cta_vec[2 + c] = sA[j * PLD + c];
        if (c == 0) cta_vec[1] = sA[j * PLD + j];
      }
      panel_sync(nclus);
      sigma = 0.f;
      for (int q = 0; q < nclus; ++q) sigma += ld_cluster_f32(&cta_vec[0], q);
      x0 = ld_cluster_f32(&cta_vec[1], 0);
      ajc = ld_cluster_f32(&cta_vec[2 + c], 0);
    }
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
    // rows of this warp strictly below row j start at tb (j < 32 <= chunk)
    const int tb = (r0 + w <= j) ? 1 : 0;
    // ---- (b) D_c = sum_{i > j} a_ij a_ic
    float dsum = 0.f;
#pragma unroll 4
    for (int li = w + QP_W * tb; li < nloc; li += QP_W) dsum += sA[li * PLD + j] * sA[li * PLD + c];
    red_dot[w * PLD + c] = dsum;
    __syncthreads();
    float dtot = 0.f;
#pragma unroll 8
    for (int q = 0; q < QP_W; ++q) dtot += red_dot[q * PLD + c];
    if (nclus > 1) {
      if (w == 0) cta_dot[c] = dtot;
      panel_sync(nclus);
      dtot = 0.f;
      for (int q = 0; q < nclus; ++q) dtot += ld_cluster_f32(&cta_dot[c], q);
    }
    const float dot = ajc + scale * dtot;  // v_j^T a_c (c > j) or v_c^T v_j (c < j)
    const float f = tau * dot;
    if (w == 0 && c < j) sG[c * PLD + j] = dot;
    // ---- (c) update below row j; column j becomes v_j; next column's sum of squares
    const float coef = c > j ? f * scale : (c == j ? 1.f - scale : 0.f);
    ss = 0.f;
#pragma unroll 4
    for (int li = w + QP_W * tb; li < nloc; li += QP_W) {
      const float aij = sA[li * PLD + j];
      const float x = sA[li * PLD + c] - coef * aij;
      __syncwarp();
      sA[li * PLD + c] = x;
      ss += (r0 + li > j + 1) ? x * x : 0.f;
    }
    if (crank == 0 && w == j && c > j) sA[j * PLD + c] -= f;  // row j: v_j(j) = 1
    if (threadIdx.x == 0) {
      sTau[j] = tau;
      sBeta[j] = beta;
    }
  }
  __syncthreads();
  // ---- T (upper): T[a][j] = -tau_j sum_{b=a}^{j-1} T[a][b] G[b][j]; lane a builds row a
  if (w == 0) {
    const int a = c;
    float trow[PB];
#pragma unroll
    for (int b = 0; b < PB; ++b) trow[b] = (b == a && a < kb) ? sTau[a] : 0.f;
#pragma unroll
    for (int j = 1; j < PB; ++j) {
      float sacc = 0.f;
#pragma unroll
      for (int b = 0; b < PB; ++b)
        if (b < j) sacc += trow[b] * sG[b * PLD + j];  // trow[b] = 0 for b < a
      if (a < j && j < kb) trow[j] = -sTau[j] * sacc;
    }
    if (crank == 0) {
#pragma unroll
      for (int b = 0; b < PB; ++b) Tg[a * PB + b] = trow[b];
    }
  }
  // ---- R block (CTA 0): upper part of rows 0..kb-1, diagonal = beta
  if (crank == 0)
    for (int e = threadIdx.x; e < kb * kb; e += QP_T) {
      const int i = e / kb, cc = e % kb;
      if (cc > i) A[(int64_t)i * n + cc] = sA[i * PLD + cc];
      if (cc == i) A[(int64_t)i * n + cc] = sBeta[i];
    }
  // ---- V: fp32 (for V^T C) and split [Vhi | Vhi | Vlo] (A operand of the 3xTF32 update)
  for (int li = w; li < nloc; li += QP_W) {
    const int gi = r0 + li;
    const float v = (c < kb) ? (gi > c ? sA[li * PLD + c] : (gi == c ? 1.f : 0.f)) : 0.f;
    Vg[(int64_t)gi * PB + c] = v;
    const float hi = tf32_hi(v);
    float* vr = Vc + (int64_t)gi * KC;
    vr[c] = hi;
    vr[PB + c] = hi;
    vr[2 * PB + c] = tf32_hi(v - hi);
  }
  if (nclus > 1) panel_sync(nclus);  // no CTA exits while others may still read its shared memory
}

// W' = T^T (V^T C) for the trailing columns C = A[j0:, j0+32:] (rows x nt),
// fp32, written split as [W'hi ; W'lo ; W'hi] (KC rows, row stride ldw).
// One CTA per (64-column tile, matrix): warp w takes rows w, w+8, ..., lane c
// columns c and c + 32 of the tile.
constexpr int QW_T = 256;
constexpr int QW_COLS = 64;
// With splits > 1 (grid.z = splits) each CTA takes one row range and writes
// its partial V^T C to Wp [b, splits, PB, nt]; qr_w_finish_kernel sums them.
__global__ void __launch_bounds__(QW_T) qr_w_kernel(const float* __restrict__ A_all, int n, int64_t bstride, int j0,
                                                  int rows, int nt, const float* __restrict__ Vg_all, int64_t vstride,
                                                  const float* __restrict__ Tg_all, float* __restrict__ Wc_all,
                                                  int64_t wstride, int ldw, int splits, float* __restrict__ Wp_all) {
  const int mat = blockIdx.y;
  const int col0 = blockIdx.x * QW_COLS;
  const int w = threadIdx.x / 32, c = threadIdx.x % 32;
  const int split = blockIdx.z;
  const int rchunk = ((rows + splits - 1) / splits + 7) / 8 * 8;
  const int r_lo = split * rchunk;
  const int r_hi = min(rows, r_lo + rchunk);
  const float* Ct = A_all + (int64_t)mat * bstride + (int64_t)j0 * n + j0 + PB + col0;
  const float* V = Vg_all + (int64_t)mat * vstride;
  const bool ok0 = col0 + c < nt, ok1 = col0 + 32 + c < nt;
  float acc0[PB], acc1[PB];
#pragma unroll
  for (int a = 0; a < PB; ++a) acc0[a] = acc1[a] = 0.f;
  // rows in batches of kRB per warp: all 2*kRB loads of the batch are issued before the FMAs
  constexpr int kRB = 8;
  int i0 = r_lo + w;
  for (; i0 + 8 * (kRB - 1) < r_hi; i0 += 8 * kRB) {
    float x0[kRB], x1[kRB];
#pragma unroll
    for (int u = 0; u < kRB; ++u) {
      x0[u] = ok0 ? Ct[(int64_t)(i0 + 8 * u) * n + c] : 0.f;
      x1[u] = ok1 ? Ct[(int64_t)(i0 + 8 * u) * n + 32 + c] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kRB; ++u) {
      const float4* vr = reinterpret_cast<const float4*>(V + (int64_t)(i0 + 8 * u) * PB);
#pragma unroll
      for (int a4 = 0; a4 < PB / 4; ++a4) {
        const float4 v4 = vr[a4];
        acc0[4 * a4 + 0] += v4.x * x0[u];
        acc0[4 * a4 + 1] += v4.y * x0[u];
        acc0[4 * a4 + 2] += v4.z * x0[u];
        acc0[4 * a4 + 3] += v4.w * x0[u];
        acc1[4 * a4 + 0] += v4.x * x1[u];
        acc1[4 * a4 + 1] += v4.y * x1[u];
        acc1[4 * a4 + 2] += v4.z * x1[u];
        acc1[4 * a4 + 3] += v4.w * x1[u];
      }
    }
  }
  for (int i = i0; i < r_hi; i += 8) {
    const float x0 = ok0 ? Ct[(int64_t)i * n + c] : 0.f;
    const float x1 = ok1 ? Ct[(int64_t)i * n + 32 + c] : 0.f;
    const float4* vr = reinterpret_cast<const float4*>(V + (int64_t)i * PB);
#pragma unroll
    for (int a4 = 0; a4 < PB / 4; ++a4) {
      const float4 v4 = vr[a4];
      acc0[4 * a4 + 0] += v4.x * x0;
      acc0[4 * a4 + 1] += v4.y * x0;
      acc0[4 * a4 + 2] += v4.z * x0;
      acc0[4 * a4 + 3] += v4.w * x0;
      acc1[4 * a4 + 0] += v4.x * x1;
      acc1[4 * a4 + 1] += v4.y * x1;
      acc1[4 * a4 + 2] += v4.z * x1;
      acc1[4 * a4 + 3] += v4.w * x1;
    }
  }
  extern __shared__ __align__(16) float wsm[];
  float* part = wsm;                     // [8][PB][QW_COLS + 1]
  float* sT = part + 8 * PB * (QW_COLS + 1);  // [PB][PLD]
  constexpr int PL = QW_COLS + 1;
#pragma unroll
  for (int a = 0; a < PB; ++a) {
    part[(w * PB + a) * PL + c] = acc0[a];
    part[(w * PB + a) * PL + 32 + c] = acc1[a];
  }
  const float* T = Tg_all + (int64_t)mat * PB * PB;
  for (int e = threadIdx.x; e < PB * PB; e += QW_T) sT[(e / PB) * PLD + e % PB] = T[e];
  __syncthreads();
  // W[b][col] summed over the 8 row groups, kept in part[0]
  for (int e = threadIdx.x; e < PB * QW_COLS; e += QW_T) {
    const int b = e / QW_COLS, col = e % QW_COLS;
    float sacc = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) sacc += part[(q * PB + b) * PL + col];
    part[b * PL + col] = sacc;  // q = 0 slot: only this thread reads or writes (b, col)
  }
  if (splits > 1) {
    float* Wp = Wp_all + ((int64_t)mat * splits + split) * PB * nt;
    for (int e = threadIdx.x; e < PB * QW_COLS; e += QW_T) {
      const int b = e / QW_COLS, col = e % QW_COLS;
      if (col0 + col < nt) Wp[(int64_t)b * nt + col0 + col] = part[b * PL + col];
    }
    return;
  }
  __syncthreads();
  float* Wc = Wc_all + (int64_t)mat * wstride;
  for (int e = threadIdx.x; e < PB * QW_COLS; e += QW_T) {
    const int a = e / QW_COLS, col = e % QW_COLS;
    if (col0 + col >= nt) continue;
    float sacc = 0.f;  // (T^T W)[a][col] = sum_{b <= a} T[b][a] W[b][col]
#pragma unroll
    for (int b = 0; b < PB; ++b)
      if (b <= a) sacc += sT[b * PLD + a] * part[b * PL + col];
    const float hi = tf32_hi(sacc);
    Wc[(int64_t)a * ldw + col0 + col] = hi;
    Wc[(int64_t)(PB + a) * ldw + col0 + col] = tf32_hi(sacc - hi);
    Wc[(int64_t)(2 * PB + a) * ldw + col0 + col] = hi;
  }
}

// W' = T^T sum_s Wp[s] for the row-split qr_w_kernel, written split like it.
__global__ void __launch_bounds__(QW_T) qr_w_finish_kernel(const float* __restrict__ Wp_all, int splits, int nt,
                                                         const float* __restrict__ Tg_all, float* __restrict__ Wc_all,
                                                         int64_t wstride, int ldw) {
  const int mat = blockIdx.y;
  const int col0 = blockIdx.x * QW_COLS;
  constexpr int PL = QW_COLS + 1;
  __shared__ float sW[PB * PL];
  __shared__ float sT[PB * PLD];
  const float* Wp = Wp_all + (int64_t)mat * splits * PB * nt;
  for (int e = threadIdx.x; e < PB * QW_COLS; e += QW_T) {
    const int b = e / QW_COLS, col = e % QW_COLS;
    float sacc = 0.f;
    if (col0 + col < nt)
      for (int q = 0; q < splits; ++q) sacc += Wp[((int64_t)q * PB + b) * nt + col0 + col];
    sW[b * PL + col] = sacc;
  }
  const float* T = Tg_all + (int64_t)mat * PB * PB;
  for (int e = threadIdx.x; e < PB * PB; e += QW_T) sT[(e / PB) * PLD + e % PB] = T[e];
  __syncthreads();
  float* Wc = Wc_all + (int64_t)mat * wstride;
  for (int e = threadIdx.x; e < PB * QW_COLS; e += QW_T) {
    const int a = e / QW_COLS, col = e % QW_COLS;
    if (col0 + col >= nt) continue;
    float sacc = 0.f;
#pragma unroll
    for (int b = 0; b < PB; ++b)
      if (b <= a) sacc += sT[b * PLD + a] * sW[b * PL + col];
    const float hi = tf32_hi(sacc);
    Wc[(int64_t)a * ldw + col0 + col] = hi;
    Wc[(int64_t)(PB + a) * ldw + col0 + col] = tf32_hi(sacc - hi);
    Wc[(int64_t)(2 * PB + a) * ldw + col0 + col] = hi;
  }
}

// R = upper triangle of A[:n, :n] (the R blocks of the panels plus the
// trailing-update results left in rows that no later panel touches).
__global__ void qr_extract_r_kernel(const float* __restrict__ A_all, int n, int64_t bstride,
                                    float* __restrict__ R_all, int64_t rstride) {
  const int mat = blockIdx.y;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)n * n) return;
  const int i = (int)(e / n), j = (int)(e % n);
  R_all[(int64_t)mat * rstride + e] = j >= i ? A_all[(int64_t)mat * bstride + (int64_t)i * n + j] : 0.f;
}

// ------------------------------------------------------------ QR panel, register-resident
// One CTA per matrix (no cluster), NW warps. Thread (w, lane) holds panel rows
// gi(u) = (u * NW + w) * 32 + lane, u < R, with all 32 panel columns in
// registers. Column step j:
//   (1) each thread forms x_ij a_ic for its rows i > j and every column c; a
//       warp transpose-reduction (32 shuffles) leaves lane c with the warp's
//       sum of column c;
//   (2) warp 0 adds the NW warp sums: D_c = sum_{i>j} x_ij a_ic. D_j is the
//       squared norm below the diagonal, so the reflector needs no separate
//       reduction; v_j^T a_c = a_jc + scale D_c is the update coefficient
//       for c > j and the entry (V^T V)_{cj} of T's input for c < j;
//   (3) each thread applies the reflector to its own rows.
// Two CTA barriers per column and no shared-memory traffic proportional to
// the panel (the shared-memory panel kernel above is bound by it). Rows:
// R = 1 up to 512 rows, R = 2 up to 1024 (512 threads), R = 3 up to 1344
// (448 threads: 144 registers for the 96 panel values).
constexpr unsigned kFullMask = 0xffffffffu;

// d[0..15] per lane -> column (lane & 15) summed over all 32 lanes
__device__ __forceinline__ float warp_colsum16(float (&d)[16], int lane) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool hi = lane & 8;
    const float send = hi ? d[k] : d[k + 8];
    const float keep = hi ? d[k + 8] : d[k];
    d[k] = keep + __shfl_xor_sync(kFullMask, send, 8);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool hi = lane & 4;
    const float send = hi ? d[k] : d[k + 4];
    const float keep = hi ? d[k + 4] : d[k];
    d[k] = keep + __shfl_xor_sync(kFullMask, send, 4);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool hi = lane & 2;
    const float send = hi ? d[k] : d[k + 2];
    const float keep = hi ? d[k + 2] : d[k];
    d[k] = keep + __shfl_xor_sync(kFullMask, send, 2);
  }
  {
    const bool hi = lane & 1;
    const float send = hi ? d[0] : d[1];
    const float keep = hi ? d[1] : d[0];
    d[0] = keep + __shfl_xor_sync(kFullMask, send, 1);
  }
  return d[0] + __shfl_xor_sync(kFullMask, d[0], 16);
}

// d[0..7] per lane -> column (lane & 7) summed over all 32 lanes
__device__ __forceinline__ float warp_colsum8(float (&d)[8], int lane) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool hi = lane & 4;
    const float send = hi ? d[k] : d[k + 4];
    const float keep = hi ? d[k + 4] : d[k];
    d[k] = keep + __shfl_xor_sync(kFullMask, send, 4);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool hi = lane & 2;
    const float send = hi ? d[k] : d[k + 2];
    const float keep = hi ? d[k + 2] : d[k];
    d[k] = keep + __shfl_xor_sync(kFullMask, send, 2);
  }
  {
    const bool hi = lane & 1;
    const float send = hi ? d[0] : d[1];
    const float keep = hi ? d[1] : d[0];
    d[0] = keep + __shfl_xor_sync(kFullMask, send, 1);
  }
  d[0] += __shfl_xor_sync(kFullMask, d[0], 8);
  return d[0] + __shfl_xor_sync(kFullMask, d[0], 16);
}

template <int R>
constexpr int qr_reg_threads() {
  return R <= 2 ? 512 : 448;  // 128 / 144 registers a thread: the R x 32 panel values
}

template <int R>
__global__ void __launch_bounds__(qr_reg_threads<R>(), 1)
    qr_panel_reg_kernel(float* __restrict__ A_all, int m, int n, int64_t bstride, int j0, int kb,
                        float* __restrict__ Vg_all, float* __restrict__ Vc_all, float* __restrict__ Tg_all,
                        int64_t vstride, int64_t cstride) {
  const int mat = blockIdx.x;
  const int rows = m - j0;
  const int NW = (int)(blockDim.x >> 5);
  const int w = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
  float* A = A_all + (int64_t)mat * bstride + (int64_t)j0 * n + j0;  // panel origin, row stride n
  __shared__ float red[32][PLD];
  __shared__ float rowj[PB];
  __shared__ float coef[PB];
  __shared__ float fj[PB];
  __shared__ float sG[PB][PLD];
  __shared__ float sTau[PB], sBeta[PB];

  float a[R][PB];
  int gi[R];
#pragma unroll
  for (int u = 0; u < R; ++u) {
    gi[u] = (u * NW + w) * 32 + lane;
    const bool ok = gi[u] < rows;
    const float4* src = reinterpret_cast<const float4*>(A + (int64_t)(ok ? gi[u] : 0) * n);
#pragma unroll
    for (int c4 = 0; c4 < PB / 4; ++c4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok && 4 * c4 < kb) v = src[c4];
      a[u][4 * c4 + 0] = v.x;
      a[u][4 * c4 + 1] = v.y;
      a[u][4 * c4 + 2] = v.z;
      a[u][4 * c4 + 3] = v.w;
    }
  }

  // The loop is rolled (a fully unrolled 32-step body overflows the
  // instruction cache); the register window rotates by one column a step so
  // that column j always sits in slot 0: slot k holds column (k + j) mod 32.
#pragma unroll 1
  for (int j = 0; j < kb; ++j) {
    // ---- (1) x_ij a_ic over this thread's rows below j; warp sums per slot
    float xj[R];
#pragma unroll
    for (int u = 0; u < R; ++u) xj[u] = gi[u] > j ? a[u][0] : 0.f;
    if (w == 0 && lane == j) {
#pragma unroll
      for (int k = 0; k < PB; ++k) rowj[k] = a[0][k];
    }
    // slot groups of GW (a transpose-reduction each; 8 wide beside a 3-row window)
    constexpr int GW = R >= 3 ? 8 : 16;
    float mine = 0.f;
#pragma unroll
    for (int h = 0; h < PB / GW; ++h) {
      float d[GW];
#pragma unroll
      for (int k = 0; k < GW; ++k) {
        float sacc = 0.f;
#pragma unroll
        for (int u = 0; u < R; ++u) sacc = fmaf(xj[u], a[u][GW * h + k], sacc);
        d[k] = sacc;
      }
      float t;
      if constexpr (GW == 16) {
        t = warp_colsum16(d, lane);
      } else {
        t = warp_colsum8(d, lane);
      }
      if (lane / GW == h) mine = t;
    }
    red[w][lane] = mine;
    __syncthreads();
    // ---- (2) reflector and coefficients (warp 0, lane = slot, column c = (lane + j) mod 32)
    if (w == 0) {
      float tot = 0.f;
      for (int q = 0; q < NW; ++q) tot += red[q][lane];
      const float sigma = __shfl_sync(kFullMask, tot, 0);
      const float x0 = rowj[0];
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
      const int c = lane + j;                  // column + 32 if it wrapped (a finished column c - 32 < j)
      const bool later = lane > 0 && c < PB;   // c > j
      const float dot = rowj[lane] + scale * tot;  // v_j^T a_c (c > j) or v_c^T v_j (c < j)
      const float f = tau * dot;
      if (c >= PB) sG[c - PB][j] = dot;
      coef[lane] = later ? f * scale : (lane == 0 ? 1.f - scale : 0.f);
      fj[lane] = later ? f : 0.f;
      if (lane == 0) {
        sTau[j] = tau;
        sBeta[j] = beta;
      }
    }
    __syncthreads();
    // ---- (3) apply to this thread's rows (slot 0 becomes v_j below the diagonal), then rotate
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const float x = a[u][0];
      if (gi[u] > j) {
#pragma unroll
        for (int k = 0; k < PB; ++k) a[u][k] = fmaf(-coef[k], x, a[u][k]);
      } else if (gi[u] == j) {
#pragma unroll
        for (int k = 1; k < PB; ++k) a[u][k] -= fj[k];
        a[u][0] = sBeta[j];
      }
      const float first = a[u][0];
#pragma unroll
      for (int k = 0; k < PB - 1; ++k) a[u][k] = a[u][k + 1];
      a[u][PB - 1] = first;
    }
  }
  // a narrow last panel (kb < 32): rotate the window back to column order
#pragma unroll 1
  for (int j = kb; j < PB; ++j) {
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const float first = a[u][0];
#pragma unroll
      for (int k = 0; k < PB - 1; ++k) a[u][k] = a[u][k + 1];
      a[u][PB - 1] = first;
    }
  }
  // ---- R block: panel rows 0..kb-1 are warp 0's first row set
  if (w == 0 && lane < kb) {
    float* Arow = A + (int64_t)lane * n;
#pragma unroll
    for (int c = 0; c < PB; ++c)
      if (c >= lane && c < kb) Arow[c] = a[0][c];
  }
  // ---- V: fp32 (for V^T C) and split [Vhi | Vhi | Vlo] (A operand of the 3xTF32 update)
  float* Vg = Vg_all + (int64_t)mat * vstride;
  float* Vc = Vc_all + (int64_t)mat * cstride;
#pragma unroll
  for (int u = 0; u < R; ++u) {
    if (gi[u] < rows) {
      float4* vg = reinterpret_cast<float4*>(Vg + (int64_t)gi[u] * PB);
      float4* vc = reinterpret_cast<float4*>(Vc + (int64_t)gi[u] * KC);
#pragma unroll
      for (int c4 = 0; c4 < PB / 4; ++c4) {
        float v[4], hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 4 * c4 + e;
          v[e] = c < kb ? (gi[u] > c ? a[u][c] : (gi[u] == c ? 1.f : 0.f)) : 0.f;
          hi[e] = tf32_hi(v[e]);
          lo[e] = tf32_hi(v[e] - hi[e]);
        }
        vg[c4] = make_float4(v[0], v[1], v[2], v[3]);
        vc[c4] = make_float4(hi[0], hi[1], hi[2], hi[3]);
        vc[PB / 4 + c4] = make_float4(hi[0], hi[1], hi[2], hi[3]);
        vc[2 * PB / 4 + c4] = make_float4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
  }
  // (after the row outputs: the panel registers are free for T's row)
  // ---- T (upper): T[a][j] = -tau_j sum_{b=a}^{j-1} T[a][b] G[b][j]; lane a builds row a
  if (w == 0) {
    const int ar = lane;
    float trow[PB];
#pragma unroll
    for (int b = 0; b < PB; ++b) trow[b] = (b == ar && ar < kb) ? sTau[ar] : 0.f;
#pragma unroll
    for (int jj = 1; jj < PB; ++jj) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int b = 0; b < jj; ++b) {
        if (b & 1) s1 = fmaf(trow[b], sG[b][jj], s1);
        else s0 = fmaf(trow[b], sG[b][jj], s0);
      }
      if (ar < jj && jj < kb) trow[jj] = -sTau[jj] * (s0 + s1);
    }
    float* Tg = Tg_all + (int64_t)mat * PB * PB;
#pragma unroll
    for (int b = 0; b < PB; ++b) Tg[ar * PB + b] = trow[b];
  }
}

// ------------------------------------------------------------ Cholesky panel
// grid (row blocks of 256, matrices). Warp 0 of every CTA factors the 32 x 32
// diagonal block in registers (left-looking: lane i holds row i, the entries
// of row j arrive by warp shuffles), then each thread solves one row of the
// panel below it, x L11^T = a, with the CTA's rows staged through shared
// memory so global loads and stores are whole rows. CTA 0 writes L11 back
// and the pivot flag.
constexpr int CP_T = 256;
__global__ void __launch_bounds__(CP_T) chol_panel_kernel(float* __restrict__ A_all, int r, int64_t bstride, int j0,
                                                        int kb, float* __restrict__ La_all,
                                                        float* __restrict__ Lb_all, int64_t lstride,
                                                        int* __restrict__ info) {
  const int mat = blockIdx.y;
  float* A = A_all + (int64_t)mat * bstride;
  __shared__ float sD[PB][PLD];
  __shared__ float sInv[PB];
  __shared__ float sRows[CP_T][PLD];
  __shared__ int bad;
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    float a[PB];
#pragma unroll
    for (int t = 0; t < PB; ++t)
      a[t] = (i < kb && t <= i) ? A[(int64_t)(j0 + i) * r + j0 + t] : (t == i ? 1.f : 0.f);
    int lbad = 0;
#pragma unroll
    for (int j = 0; j < PB; ++j) {
      float sacc = a[j];
#pragma unroll
      for (int t = 0; t < PB; ++t) {
        if (t < j) {
          const float ljt = __shfl_sync(0xffffffffu, a[t], j);
          sacc -= a[t] * ljt;
        }
      }
      float piv = sacc;
      if (i == j && !(piv > 0.f)) {
        lbad = 1;
        piv = __int_as_float(0x7fc00000);  // NaN: the caller's guard discards this matrix
      }
      const float ljj = __shfl_sync(0xffffffffu, sqrtf(piv), j);
      if (i > j) a[j] = sacc / ljj;
      if (i == j) a[j] = ljj;
    }
    float dg = 1.f;
#pragma unroll
    for (int t = 0; t < PB; ++t) {
      sD[i][t] = t <= i ? a[t] : 0.f;
      if (t == i) dg = a[t];  // static indices keep a[] in registers
    }
    sInv[i] = 1.f / dg;
    const int anybad = __any_sync(0xffffffffu, lbad && i < kb);
    if (i == 0) bad = anybad;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < kb * kb; e += CP_T) {
      const int i = e / kb, j = e % kb;
      if (j <= i) A[(int64_t)(j0 + i) * r + j0 + j] = sD[i][j];
    }
    if (threadIdx.x == 0 && bad && info != nullptr) info[mat] = 1;
  }
  const int rows = r - j0 - kb;
  const int row0 = blockIdx.x * CP_T;
  const int nr = min(CP_T, rows - row0);
  if (nr <= 0) return;
  for (int e = threadIdx.x; e < nr * PB; e += CP_T) {
    const int i = e / PB, j = e % PB;
    sRows[i][j] = j < kb ? A[(int64_t)(j0 + kb + row0 + i) * r + j0 + j] : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < nr) {
    float x[PB];
#pragma unroll
    for (int j = 0; j < PB; ++j) x[j] = sRows[threadIdx.x][j];
#pragma unroll
    for (int j = 0; j < PB; ++j) {
      float sacc = x[j];
#pragma unroll
      for (int t = 0; t < PB; ++t)
        if (t < j) sacc -= x[t] * sD[j][t];
      x[j] = j < kb ? sacc * sInv[j] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < PB; ++j) sRows[threadIdx.x][j] = x[j];
  }
  __syncthreads();
  float* la = La_all + (int64_t)mat * lstride + (int64_t)row0 * KC;
  float* lb = Lb_all + (int64_t)mat * lstride + (int64_t)row0 * KC;
  for (int e = threadIdx.x; e < nr * PB; e += CP_T) {
    const int i = e / PB, j = e % PB;
    const float v = sRows[i][j];
    if (j < kb) A[(int64_t)(j0 + kb + row0 + i) * r + j0 + j] = v;
    const float hi = tf32_hi(v);
    const float lo = tf32_hi(v - hi);
    la[(int64_t)i * KC + j] = hi;
    la[(int64_t)i * KC + PB + j] = hi;
    la[(int64_t)i * KC + 2 * PB + j] = lo;
    lb[(int64_t)i * KC + j] = hi;
    lb[(int64_t)i * KC + PB + j] = lo;
    lb[(int64_t)i * KC + 2 * PB + j] = hi;
  }
}

}  // namespace

// A: [b, m, n] fp32 contiguous (m >= n, n % 4 == 0), overwritten; R: [b, n, n] upper.
void qr_r_blocked(at::Tensor& A, at::Tensor& R) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) >= A.size(2),
              "dion_b200 qr_r_blocked: contiguous [b, m, n] fp32 with m >= n");
  TORCH_CHECK(A.size(2) % 4 == 0, "dion_b200 qr_r_blocked: n must be a multiple of 4 (16-byte rows)");
  TORCH_CHECK(R.is_contiguous() && R.size(0) == A.size(0) && R.size(1) == A.size(2) && R.size(2) == A.size(2),
              "dion_b200 qr_r_blocked: R must be a contiguous [b, n, n] tensor");
  const int b = (int)A.size(0), m = (int)A.size(1), n = (int)A.size(2);
  if (b == 0 || A.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  TORCH_CHECK((int64_t)m <= 8LL * kQrMaxChunk, "dion_b200 qr_r_blocked: m too large (at most 8 x 1400 rows)");
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t bs = (int64_t)m * n;
  auto opt = A.options();
  // rows of a panel per CTA (more rows: a cluster of 2, 4 or 8 CTAs shares the panel);
  // DION_B200_QR_CHUNK lowers it to trade per-CTA work for cluster barriers
  static const int max_chunk = [] {
    const char* e = std::getenv("DION_B200_QR_CHUNK");
    const int v = e ? std::atoi(e) : kQrDefaultChunk;
    return std::max(64, std::min(kQrMaxChunk, v));
  }();
  at::Tensor Vg = at::empty({b, m, PB}, opt);
  at::Tensor Vc = at::empty({b, m, KC}, opt);
  at::Tensor Tg = at::empty({b, PB, PB}, opt);
  at::Tensor Wc = at::empty({b, KC, n}, opt);
  constexpr size_t w_smem = (size_t)(8 * PB * (QW_COLS + 1) + PB * PLD) * sizeof(float);
  static bool w_attr = false;
  if (!w_attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(qr_w_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)w_smem));
    w_attr = true;
  }
  // panels of up to 1536 rows: the register-resident kernel (one CTA per matrix);
  // DION_B200_QR_PANEL=smem keeps the shared-memory / cluster kernel throughout
  static const bool reg_panels = [] {
    const char* e = std::getenv("DION_B200_QR_PANEL");
    return !(e && std::string(e) == "smem");
  }();
  // W' row splits: about two CTAs per SM over the batch (decided per panel, at most splits_max)
  const int splits_max = std::max(1, std::min(8, (2 * 148) / b + 1));
  at::Tensor Wp = splits_max > 1 ? at::empty({b, splits_max, PB, n}, opt) : at::Tensor();
  for (int j0 = 0; j0 < n; j0 += PB) {
    const int kb = std::min(PB, n - j0);
    const int rows = m - j0;
    const int R = !reg_panels ? 0 : rows <= 512 ? 1 : rows <= 1024 ? 2 : rows <= 1344 ? 3 : 0;
    if (R > 0) {
      const int nw = (rows + 32 * R - 1) / (32 * R);
      const dim3 grid((unsigned)b), block((unsigned)(32 * nw));
      float* Ap = A.data_ptr<float>();
      if (R == 1)
        qr_panel_reg_kernel<1><<<grid, block, 0, stream>>>(Ap, m, n, bs, j0, kb, Vg.data_ptr<float>(),
                                                           Vc.data_ptr<float>(), Tg.data_ptr<float>(),
                                                           (int64_t)m * PB, (int64_t)m * KC);
      else if (R == 2)
        qr_panel_reg_kernel<2><<<grid, block, 0, stream>>>(Ap, m, n, bs, j0, kb, Vg.data_ptr<float>(),
                                                           Vc.data_ptr<float>(), Tg.data_ptr<float>(),
                                                           (int64_t)m * PB, (int64_t)m * KC);
      else
        qr_panel_reg_kernel<3><<<grid, block, 0, stream>>>(Ap, m, n, bs, j0, kb, Vg.data_ptr<float>(),
                                                           Vc.data_ptr<float>(), Tg.data_ptr<float>(),
                                                           (int64_t)m * PB, (int64_t)m * KC);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      note_launch();
    } else {
    int nclus = 1;
    while ((rows + nclus - 1) / nclus > max_chunk && nclus < 8) nclus *= 2;
    const int chunk = (rows + nclus - 1) / nclus;
    const size_t smem = ((size_t)chunk * PLD + QP_W + QP_W * PLD + 2 + 2 * PB + PB * PLD + 2 * PB) * sizeof(float);
    C10_CUDA_CHECK(cudaFuncSetAttribute(qr_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(b * nclus));
    cfg.blockDim = dim3(QP_T);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)nclus;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, qr_panel_kernel, A.data_ptr<float>(), m, n, bs, j0, kb, chunk,
                                      Vg.data_ptr<float>(), Vc.data_ptr<float>(), Tg.data_ptr<float>(),
                                      (int64_t)m * PB, (int64_t)m * KC, nclus));
    note_launch();
    }
    const int nt = n - j0 - kb;
    if (nt <= 0) continue;
    const int ntiles = (nt + QW_COLS - 1) / QW_COLS;
    const int splits = std::max(1, std::min({splits_max, (2 * 148) / (ntiles * b) + 1, rows / 256}));
    qr_w_kernel<<<dim3((unsigned)ntiles, (unsigned)b, (unsigned)splits), QW_T, w_smem, stream>>>(
        A.data_ptr<float>(), n, bs, j0, rows, nt, Vg.data_ptr<float>(), (int64_t)m * PB, Tg.data_ptr<float>(),
        Wc.data_ptr<float>(), (int64_t)KC * n, n, splits, splits > 1 ? Wp.data_ptr<float>() : nullptr);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    if (splits > 1) {
      qr_w_finish_kernel<<<dim3((unsigned)ntiles, (unsigned)b), QW_T, 0, stream>>>(
          Wp.data_ptr<float>(), splits, nt, Tg.data_ptr<float>(), Wc.data_ptr<float>(), (int64_t)KC * n, n);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      note_launch();
    }
    // A[j0:, j0+32:] -= [Vhi|Vhi|Vlo] [W'hi;W'lo;W'hi]   (tcgen05, in place)
    at::Tensor Vsub = Vc.narrow(1, 0, rows);
    at::Tensor Wsub = Wc.narrow(2, 0, nt);
    at::Tensor Csub = A.narrow(1, j0, rows).narrow(2, j0 + kb, nt);
    gemm_ex(Vsub, Wsub, Csub, Csub, -1.0, 1.0, c10::nullopt, 0, 0, false, false, 1.0, 1.0, 0, c10::nullopt, 0, 0, 1,
            0, 0, 0);
  }
  const int64_t nn = (int64_t)n * n;
  qr_extract_r_kernel<<<dim3((unsigned)((nn + 255) / 256), (unsigned)b), 256, 0, stream>>>(
      A.data_ptr<float>(), n, bs, R.data_ptr<float>(), nn);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  note_launch();
}

// A: [b, r, r] fp32 contiguous (r % 4 == 0), overwritten with L in its lower
// triangle (the strict upper triangle is left with scratch values); info[b]
// int32 = 1 where a pivot was not positive.
void cholesky_blocked(at::Tensor& A, at::Tensor& info) {
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.scalar_type() == at::kFloat && A.size(1) == A.size(2),
              "dion_b200 cholesky_blocked: contiguous [b, r, r] fp32");
  TORCH_CHECK(A.size(1) % 4 == 0, "dion_b200 cholesky_blocked: r must be a multiple of 4 (16-byte rows)");
  TORCH_CHECK(info.scalar_type() == at::kInt && info.numel() >= A.size(0) && info.is_cuda(),
              "dion_b200 cholesky_blocked: info must be an int32 CUDA tensor of b entries");
  const int b = (int)A.size(0), r = (int)A.size(1);
  if (b == 0 || A.numel() == 0) return;  // nothing to do (e.g. a rank that holds no matrix of a batch)
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(info.data_ptr<int>(), 0, sizeof(int) * (size_t)b, stream));
  const int64_t bs = (int64_t)r * r;
  auto opt = A.options();
  at::Tensor La = at::empty({b, r, KC}, opt);
  at::Tensor Lb = at::empty({b, r, KC}, opt);
  for (int j0 = 0; j0 < r; j0 += PB) {
    const int kb = std::min(PB, r - j0);
    const int rows = r - j0 - kb;
    const int gx = std::max(1, (rows + CP_T - 1) / CP_T);
    chol_panel_kernel<<<dim3((unsigned)gx, (unsigned)b), CP_T, 0, stream>>>(
        A.data_ptr<float>(), r, bs, j0, kb, La.data_ptr<float>(), Lb.data_ptr<float>(), (int64_t)r * KC,
        info.data_ptr<int>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    note_launch();
    if (rows <= 0) continue;
    // A22 -= L21 L21^T (symmetric mode: upper tiles computed and mirrored, in place)
    at::Tensor Lsa = La.narrow(1, 0, rows);
    at::Tensor Lsb = Lb.narrow(1, 0, rows).transpose(1, 2);
    at::Tensor A22 = A.narrow(1, j0 + kb, rows).narrow(2, j0 + kb, rows);
    gemm_ex(Lsa, Lsb, A22, A22, -1.0, 1.0, c10::nullopt, 0, 0, true, false, 1.0, 1.0, 0, c10::nullopt, 0, 0, 1, 0,
            0, 0);
  }
}

}  // namespace bdion

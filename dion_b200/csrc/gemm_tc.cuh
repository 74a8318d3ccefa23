// Persistent, warp-specialised GEMM on the sm_100a tensor cores: bf16
// operands (kind::f16) or fp32 operands on the tf32 path (kind::tf32), fp32
// accumulation in TMEM.
//
//   D[b] = epilogue( alpha_b * A[b] @ B[b] , C[b] )
//
// A[b] is M x K and B[b] is K x N; each operand may be stored K-major or
// MN-major (the layout is chosen through the TMA tensor map and the UMMA
// shared-memory descriptor, never by a transpose copy).
//
// Roles (192 threads, one CTA per SM):
//   warp 0      : TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..5  : epilogue, one TMEM lane quarter each (tcgen05.ld -> regs ->
//                 fused math -> st.global)
// The accumulator is double buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Epilogue modes:
//   store   : D = alpha_b*acc + beta_b*C
//   sym     : same, but only tiles touching the upper triangle are computed;
//             each element (i,j), j>i, is also written to (j,i). Used for the
//             symmetric products X X^T and A A of Newton-Schulz.
//   PARAM   : D = gamma*D + delta*(alpha_b*acc + beta_b*C)  (in-place weight
//             update fused into the last Newton-Schulz GEMM)
//
// Pointer-array outputs (D_ptrs): destination d of row `row` of batch b is
// D_ptrs[(b*splits + row/rows_per_ptr)*nrep + rep], rep < nrep, at local row
// row % rows_per_ptr. The addresses may be another GPU's memory (peer
// mapping): the epilogue then stores the tile over NVLink while the tensor
// cores work on the next tile, which is how GEMM -> reduce-scatter,
// GEMM -> all-gather (nrep = world) and NS -> scatter are fused.
//
// alpha_b = alpha * scale[b]^alpha_pow, beta_b = beta * scale[b]^beta_pow when
// a per-batch scale vector is given (used to fold the Frobenius
// normalisation of Newton-Schulz into the first iteration).
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace bdion {

struct GemmArgs {
  int M, N, K, batch;
  void* D;
  void* const* D_ptrs;  // optional output pointers (device array), see below
  int nrep;             // D_ptrs: copies of every output element (>= 1)
  int rows_per_ptr;     // D_ptrs: rows per destination (0: all M rows)
  int splits;           // D_ptrs: destinations per batch along M
  int64_t ldd, strideD;
  const void* C;  // may be null
  int64_t ldc, strideC;
  float alpha, beta;
  const float* scale;  // per-batch scale (may be null)
  int alpha_pow, beta_pow;
  float gamma, delta;  // PARAM mode
  int sym;
  int tiles_m, tiles_n;
  int tiles_per_batch;
  int total_tiles;
  int* status;
  uint64_t limit_ns;
  // tile-order rotation (non-symmetric GEMMs): batch b is processed as
  // (b + rot_b) % batch and row tile tm as (tm + rot_rows / BM) % tiles_m, so
  // that ranks storing to peer GPUs start on different destinations
  int rot_b;
  int rot_rows;
};

constexpr int kBM = 128;
constexpr int kGroupM = 8;

// Per-input-type constants: one K block is one 128-byte swizzle row.
template <typename TIn>
struct InCfg;
template <>
struct InCfg<__nv_bfloat16> {
  static constexpr int kBK = 64;      // elements per 128-byte row
  static constexpr int kUmmaK = 16;   // K per tcgen05.mma
  static constexpr uint32_t kFmt = 1; // bf16
  static constexpr bool kTf32 = false;
};
template <>
struct InCfg<float> {
  static constexpr int kBK = 32;
  static constexpr int kUmmaK = 8;
  static constexpr uint32_t kFmt = 2; // tf32
  static constexpr bool kTf32 = true;
};

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr int kABytes = kBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  // epilogue staging: one 32 x 33 fp32 transpose tile per epilogue warp
  static constexpr int kStagingBytes = 4 * 32 * 33 * 4;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ + kStagingBytes;
};

__device__ __forceinline__ int sym_row_start(int tm, int BN) { return (tm * kBM) / BN; }

template <int BN>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int local, int& tm, int& tn);

// tile t -> (batch, row tile, column tile) including the rotations
template <int BN>
__device__ __forceinline__ void map_tile(const GemmArgs& a, int t, int& b, int& tm, int& tn) {
  b = t / a.tiles_per_batch;
  decode_tile<BN>(a, t - b * a.tiles_per_batch, tm, tn);
  if (!a.sym) {
    if (a.rot_b) b = (b + a.rot_b) % a.batch;
    if (a.rot_rows) tm = (tm + a.rot_rows / kBM) % a.tiles_m;
  }
}

// Map a linear tile id inside one batch to (tm, tn).
template <int BN>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int local, int& tm, int& tn) {
  if (a.sym) {
    int r = 0;
    while (true) {
      int cnt = a.tiles_n - sym_row_start(r, BN);
      if (local < cnt || r == a.tiles_m - 1) {
        tm = r;
        tn = sym_row_start(r, BN) + local;
        return;
      }
      local -= cnt;
      ++r;
    }
  }
  const int per_group = kGroupM * a.tiles_n;
  const int g = local / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(a.tiles_m - first_m, kGroupM);
  const int in_g = local - g * per_group;
  tm = first_m + in_g % gsize;
  tn = in_g / gsize;
}

template <typename TIn, int BN, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  using IC = InCfg<TIn>;
  constexpr int S = Cfg::kStages;
  constexpr int kBK = IC::kBK;
  constexpr int kBoxBytes = kBK * 128;           // one MN-major box: kBK MN elems x kBK K rows
  constexpr int kKStepMN = IC::kUmmaK * 128;      // MN-major: K advance per MMA (rows x 128 B)
  // MN-major smem layout: bf16 uses the 128B swizzle (8-row atoms, SBO 1024);
  // tf32 must use the 128B swizzle with 32B atoms (4-row atoms, SBO 512).
  constexpr uint32_t kMNLayout = IC::kTf32 ? 1u : 2u;
  constexpr uint32_t kMNSbo = IC::kTf32 ? 512u : 1024u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* tfull_bar = bars + 2 * S;
  uint64_t* tempty_bar = bars + 2 * S + 2;
  uint64_t* drain_bar = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * S + 6);
  float* staging = reinterpret_cast<float*>(smem + S * Cfg::kStageBytes + 256);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 4);
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (args.K + IC::kBK - 1) / IC::kBK;
  const uint64_t limit = args.limit_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.total_tiles && ok; t += gridDim.x) {
        int b, tm, tn;
        map_tile<BN>(args, t, b, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, s_abort, limit)) {
            report_status(args.status, kStatusGemmProducerTimeout);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          if (!A_MN) {
            tma_load_3d(&tmA, &full_bar[stage], a_dst, kb * kBK, tm * kBM, b);
          } else {
#pragma unroll
            for (int h = 0; h < kBM / kBK; ++h)
              tma_load_3d(&tmA, &full_bar[stage], a_dst + h * kBoxBytes, tm * kBM + h * kBK, kb * kBK, b);
          }
          if (!B_MN) {
            tma_load_3d(&tmB, &full_bar[stage], b_dst, kb * kBK, tn * BN, b);
          } else {
#pragma unroll
            for (int h = 0; h < BN / kBK; ++h)
              tma_load_3d(&tmB, &full_bar[stage], b_dst + h * kBoxBytes, tn * BN + h * kBK, kb * kBK, b);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for the loads of the last S issued stages.
        int st = stage;
        uint32_t ph = phase;
        for (long i = 0; i < min(issued, (long)S); ++i) {
          if (--st < 0) {
            st = S - 1;
            ph ^= 1;
          }
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[st], ph) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(kBM, BN, A_MN, B_MN, IC::kFmt);
      int stage = 0;
      uint32_t phase = 0;
      int local_tile = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = blockIdx.x; t < args.total_tiles && ok; t += gridDim.x, ++local_tile) {
        const int acc = local_tile & 1;
        const uint32_t acc_phase = (local_tile >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, s_abort, limit)) {
          report_status(args.status, kStatusGemmMmaTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, s_abort, limit)) {
            report_status(args.status, kStatusGemmMmaTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / IC::kUmmaK; ++k) {
            const uint64_t adesc = A_MN ? make_sdesc_sw128(a_base + k * kKStepMN, kBoxBytes, kMNSbo, kMNLayout)
                                        : make_sdesc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sdesc_sw128(b_base + k * kKStepMN, kBoxBytes, kMNSbo, kMNLayout)
                                        : make_sdesc_sw128(b_base + k * 32, 16, 1024);
            if (IC::kTf32)
              umma_tf32(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
      }
      if (!ok && issued_any) {
        // Wait (bounded) for the MMAs already issued before TMEM is freed.
        umma_commit(drain_bar);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local_tile = 0;
    for (int t = blockIdx.x; t < args.total_tiles; t += gridDim.x, ++local_tile) {
      int b, tm, tn;
      map_tile<BN>(args, t, b, tm, tn);
      const int acc = local_tile & 1;
      const uint32_t acc_phase = (local_tile >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, s_abort, limit)) {
        report_status(args.status, kStatusGemmEpilogueTimeout);
        break;
      }
      tc_fence_after();

      float alpha = args.alpha, beta = args.beta;
      if (args.scale != nullptr) {
        const float s = args.scale[b];
        for (int i = 0; i < args.alpha_pow; ++i) alpha *= s;
        for (int i = 0; i < args.beta_pow; ++i) beta *= s;
      }
      const int row = tm * kBM + q * 32 + lane;
      const bool row_ok = row < args.M;
      int lrow = row;
      void* const* dps = nullptr;
      OutT* Db = reinterpret_cast<OutT*>(args.D) + (int64_t)b * args.strideD;
      if (args.D_ptrs != nullptr && row_ok) {
        int split = 0;
        if (args.rows_per_ptr > 0) {
          split = row / args.rows_per_ptr;
          lrow = row - split * args.rows_per_ptr;
        }
        dps = args.D_ptrs + ((int64_t)b * args.splits + split) * args.nrep;
        Db = reinterpret_cast<OutT*>(dps[0]);
      }
      const CT* Cb = args.C ? reinterpret_cast<const CT*>(args.C) + (int64_t)b * args.strideC : nullptr;

      float* stg = staging + q * (32 * 33);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, r);
        tmem_wait_ld();
        const int col0 = tn * BN + c * 32;
        if (col0 >= args.N) continue;  // warp-uniform
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = alpha * __uint_as_float(r[i]);
        const bool full = col0 + 32 <= args.N;
        if (!PARAM && !args.sym && full) {
          // Coalesced store: stage the warp's 32x32 block in shared memory, then
          // each store instruction writes whole 128-byte (fp32) / 64-byte (bf16)
          // row segments, which matters most when the rows live on a peer GPU.
          if (row_ok && Cb != nullptr && beta != 0.f) {
            const CT* crow = Cb + (int64_t)row * args.ldc + col0;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float cv[8];
              load8(crow + i, cv);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i + j] += beta * cv[j];
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) stg[lane * 33 + i] = v[i];
          __syncwarp();
          constexpr int kVec = 16 / sizeof(OutT);     // elements per 16-byte store
          constexpr int kLanesPerRow = 32 / kVec;     // 8 (fp32) or 4 (bf16)
          constexpr int kRowsPerPass = 32 / kLanesPerRow;
          const int sub = lane % kLanesPerRow;
#pragma unroll
          for (int pass = 0; pass < 32 / kRowsPerPass; ++pass) {
            const int rr = pass * kRowsPerPass + lane / kLanesPerRow;
            const int grow = tm * kBM + q * 32 + rr;
            if (grow < args.M) {
              float vals[kVec];
#pragma unroll
              for (int j = 0; j < kVec; ++j) vals[j] = stg[rr * 33 + sub * kVec + j];
              int lr = grow;
              void* const* rp = nullptr;
              OutT* base = reinterpret_cast<OutT*>(args.D) + (int64_t)b * args.strideD;
              if (args.D_ptrs != nullptr) {
                int split = 0;
                if (args.rows_per_ptr > 0) {
                  split = grow / args.rows_per_ptr;
                  lr = grow - split * args.rows_per_ptr;
                }
                rp = args.D_ptrs + ((int64_t)b * args.splits + split) * args.nrep;
                base = reinterpret_cast<OutT*>(rp[0]);
              }
              for (int rep = 0; rep < args.nrep; ++rep) {
                if (rep > 0) base = reinterpret_cast<OutT*>(rp[rep]);
                store8or4(base + (int64_t)lr * args.ldd + col0 + sub * kVec, vals);
              }
            }
          }
          __syncwarp();
          continue;
        }
        if (!row_ok) continue;
        if (Cb != nullptr && beta != 0.f) {
          const CT* crow = Cb + (int64_t)row * args.ldc + col0;
          if (full) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float cv[8];
              load8(crow + i, cv);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i + j] += beta * cv[j];
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < args.N) v[i] += beta * to_f<CT>(crow[i]);
          }
        }
        OutT* drow = Db + (int64_t)lrow * args.ldd + col0;
        if (PARAM) {
          if (full) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float pv[8];
              load8(drow + i, pv);
#pragma unroll
              for (int j = 0; j < 8; ++j) pv[j] = args.gamma * pv[j] + args.delta * v[i + j];
              store8(drow + i, pv);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < args.N) drow[i] = from_f<OutT>(args.gamma * to_f<OutT>(drow[i]) + args.delta * v[i]);
          }
        } else if (!args.sym) {
          for (int rep = 0; rep < args.nrep; ++rep) {
            if (rep > 0) drow = reinterpret_cast<OutT*>(dps[rep]) + (int64_t)lrow * args.ldd + col0;
            if (full) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) store8(drow + i, v + i);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col0 + i < args.N) drow[i] = from_f<OutT>(v[i]);
            }
          }
        } else {
          // symmetric: write (row, j) for j >= row and mirror (j, row) for j > row
          if (col0 > row && full) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) store8(drow + i, v + i);
#pragma unroll
            for (int i = 0; i < 32; ++i) Db[(int64_t)(col0 + i) * args.ldd + row] = from_f<OutT>(v[i]);
          } else if (col0 + 31 >= row) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int j = col0 + i;
              if (j >= args.N || j < row) continue;
              drow[i] = from_f<OutT>(v[i]);
              if (j > row) Db[(int64_t)j * args.ldd + row] = from_f<OutT>(v[i]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace bdion

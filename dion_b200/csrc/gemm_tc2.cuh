// CTA-pair (cta_group::2) variant of the persistent tcgen05 GEMM in
// gemm_tc.cuh: a cluster of two CTAs computes one 256 x BN tile with a
// single tcgen05.mma of M = 256 issued by the even CTA ("leader").
//
//   * each CTA TMA-loads its own half of the operands into its own shared
//     memory (A: its 128 rows; B: its BN/2 columns), without multicast; the
//     loads count their bytes on the leader's full barrier;
//   * the leader's MMA warp waits on that barrier, issues the MMAs (reading
//     both CTAs' shared memory) and commits to the empty / TMEM-full
//     barriers of both CTAs at once (multicast commit);
//   * each CTA's epilogue reads the 128 accumulator rows of its own TMEM and
//     arrives on the leader's TMEM-empty barrier;
//   * a cluster barrier precedes the paired TMEM deallocation.
// Per CTA this halves the B traffic and shared-memory footprint of a
// 128 x BN tile, which buys two more pipeline stages.
//
// Epilogue modes and arguments are those of gemm_tc.cuh (GemmArgs); every
// wait is bounded the same way.
#pragma once
#include "gemm_tc.cuh"

namespace bdion {

constexpr int kBM2 = 256;  // rows per CTA pair

template <int BN>
struct GemmCfg2 {
  static constexpr int kABytes = 128 * 128;        // 128 rows x one 128-byte K row
  static constexpr int kBBytes = (BN / 2) * 128;   // BN/2 columns
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN >= 256 ? 6 : 8;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kStagingBytes = 4 * 32 * 33 * 4;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kStagingBytes;
};

template <int BN>
__device__ __forceinline__ void decode_tile2(const GemmArgs& a, int local, int& tm, int& tn) {
  if (a.sym) {
    int r = 0;
    while (true) {
      const int start = (r * kBM2) / BN;
      int cnt = a.tiles_n - start;
      if (local < cnt || r == a.tiles_m - 1) {
        tm = r;
        tn = start + local;
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

template <int BN>
__device__ __forceinline__ void map_tile2(const GemmArgs& a, int t, int& b, int& tm, int& tn) {
  b = t / a.tiles_per_batch;
  decode_tile2<BN>(a, t - b * a.tiles_per_batch, tm, tn);
  if (!a.sym) {
    if (a.rot_b) b = (b + a.rot_b) % a.batch;
    if (a.rot_rows) tm = (tm + a.rot_rows / kBM2) % a.tiles_m;
  }
}

template <typename TIn, int BN, bool A_MN, bool B_MN, typename OutT, typename CT, bool PARAM>
__global__ void __launch_bounds__(192, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmArgs args) {
  using Cfg = GemmCfg2<BN>;
  using IC = InCfg<TIn>;
  constexpr int S = Cfg::kStages;
  constexpr int kBK = IC::kBK;
  constexpr int kBoxBytes = kBK * 128;
  constexpr int kKStepMN = IC::kUmmaK * 128;
  constexpr uint32_t kMNLayout = IC::kTf32 ? 1u : 2u;
  constexpr uint32_t kMNSbo = IC::kTf32 ? 512u : 1024u;
  constexpr int kHalfN = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full_bar = bars;              // used in the leader
  uint64_t* empty_bar = bars + S;         // both CTAs
  uint64_t* tfull_bar = bars + 2 * S;     // both CTAs
  uint64_t* tempty_bar = bars + 2 * S + 2;  // used in the leader (8 arrivals: 4 warps x 2 CTAs)
  uint64_t* drain_bar = bars + 2 * S + 4;  // leader: completion of the MMAs issued before an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * S + 6);
  float* staging = reinterpret_cast<float*>(smem + S * Cfg::kStageBytes + 256);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t crank = cluster_ctarank();
  const uint32_t half = crank & 1u;          // 0: leader, 1: peer
  const uint32_t leader = crank & ~1u;
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 8);
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
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_barrier_sync();  // both CTAs' barriers initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (args.K + kBK - 1) / kBK;
  const uint64_t limit = args.limit_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      long issued = 0;
      for (int t = pair; t < args.total_tiles && ok; t += npairs) {
        int b, tm, tn;
        map_tile2<BN>(args, t, b, tm, tn);
        const int row0 = tm * kBM2 + (int)half * 128;
        const int col0 = tn * BN + (int)half * kHalfN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, s_abort, limit)) {
            report_status(args.status, kStatusGemmProducerTimeout);
            ok = false;
            break;
          }
          if (half == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::kStageBytes);
          const uint32_t lbar = mapa_shared(smem_u32(&full_bar[stage]), leader);
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          if (!A_MN) {
            tma_load_3d_pair(&tmA, lbar, a_dst, kb * kBK, row0, b);
          } else {
#pragma unroll
            for (int h = 0; h < 128 / kBK; ++h)
              tma_load_3d_pair(&tmA, lbar, a_dst + h * kBoxBytes, row0 + h * kBK, kb * kBK, b);
          }
          if (!B_MN) {
            tma_load_3d_pair(&tmB, lbar, b_dst, kb * kBK, col0, b);
          } else {
#pragma unroll
            for (int h = 0; h < kHalfN / kBK; ++h)
              tma_load_3d_pair(&tmB, lbar, b_dst + h * kBoxBytes, col0 + h * kBK, kb * kBK, b);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && half == 0) {
        // Drain: both CTAs' loads of a stage complete on the leader's full barrier (its
        // expect_tx counts both halves), so the leader waits (bounded) for the phases of
        // the last S stages it armed. The peer CTA cannot wait on a remote barrier; it is
        // held at the final cluster barrier until this drain is over.
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
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && half == 0) {
      constexpr uint32_t idesc = make_idesc(kBM2, BN, A_MN, B_MN, IC::kFmt);
      int stage = 0;
      uint32_t phase = 0;
      int local_tile = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = pair; t < args.total_tiles && ok; t += npairs, ++local_tile) {
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
              umma_tf32_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(&empty_bar[stage], (uint16_t)(3u << leader));
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[acc], (uint16_t)(3u << leader));
      }
      if (!ok && issued_any) {
        // Wait (bounded) for the MMAs already issued before TMEM is released: a commit
        // to the leader's own drain barrier arrives once all of them have completed.
        umma_commit_pair(drain_bar, (uint16_t)(1u << leader));
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const uint32_t l_tempty0 = mapa_shared(smem_u32(&tempty_bar[0]), leader);
    const uint32_t l_tempty1 = mapa_shared(smem_u32(&tempty_bar[1]), leader);
    float* stg = staging + q * (32 * 33);
    int local_tile = 0;
    for (int t = pair; t < args.total_tiles; t += npairs, ++local_tile) {
      int b, tm, tn;
      map_tile2<BN>(args, t, b, tm, tn);
      const int acc = local_tile & 1;
      const uint32_t acc_phase = (local_tile >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, s_abort, limit)) {
        report_status(args.status, kStatusGemmEpilogueTimeout);
        break;
      }
      tc_fence_after();

      float alpha = args.alpha, beta = args.beta;
      if (args.scale != nullptr) {
        const float sc = args.scale[b];
        for (int i = 0; i < args.alpha_pow; ++i) alpha *= sc;
        for (int i = 0; i < args.beta_pow; ++i) beta *= sc;
      }
      const int rbase = tm * kBM2 + (int)half * 128;
      const int row = rbase + q * 32 + lane;
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
          constexpr int kVec = 16 / sizeof(OutT);
          constexpr int kLanesPerRow = 32 / kVec;
          constexpr int kRowsPerPass = 32 / kLanesPerRow;
          const int sub = lane % kLanesPerRow;
#pragma unroll
          for (int pass = 0; pass < 32 / kRowsPerPass; ++pass) {
            const int rr = pass * kRowsPerPass + lane / kLanesPerRow;
            const int grow = rbase + q * 32 + rr;
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
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < args.N) drow[i] = from_f<OutT>(v[i]);
          }
        } else {
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
      if (lane == 0) mbar_arrive_remote(acc ? l_tempty1 : l_tempty0);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_barrier_sync();  // both CTAs done with TMEM and with each other's shared memory
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

}  // namespace bdion

// gemm_pair.cuh — CTA-pair (cta_group::2) tcgen05 GEMM for sm_100a, normal orientation:
// D[M][N] = A[M][K] . B[N][K]^T with A = activations [tokens][K], B = weights [features][K].
//
// A cluster of two CTAs owns a 256 x 256 output tile.  Each CTA stages 128 rows of A (its half of M)
// and 128 rows of B (its half of N) per 64-wide K block; one thread of the even CTA issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads both CTAs' shared memory and writes each
// CTA's own 128 TMEM lanes x 256 columns.  Per MAC this moves a third fewer bytes from L2 into shared
// memory, and reads a third fewer from shared memory into the tensor cores, than a 128 x 256 tile on
// one SM.  Warp roles (both CTAs):
//   warp 0  TMA producer (lane 0): the CTA's own A and B halves into a STAGES-deep ring; no multicast
//   warp 1  even CTA: MMA issuer.  Odd CTA: relay — once its own stage has landed it arrives on the
//           even CTA's pair barrier for that stage, so the issuer knows both halves are in place
//   warp 2  TMEM: 2 x 256 f32 columns (double-buffered accumulator), allocated as a pair
//   warps 4-11 epilogue of the CTA's 128 rows (the same fused epilogues as gemm_tc_kernel): two warps
//           per 32-lane TMEM quarter, one per 128-column half; the accumulator is handed back to the
//           issuer with 8 local + 8 remote arrivals
// The issuer's commits are multicast to both CTAs (stage released, accumulator complete).  The per-stage
// waits are CTA-scope (acquire.cluster on every stage halved the throughput, measured) and the relay's
// arrival is relaxed: it only forwards a completion the TMA already signalled.  Every wait is bounded;
// both CTAs meet at a final cluster barrier before the TMEM is freed, after the issuer's last commit has
// landed, so neither CTA leaves while the pair's MMAs can still touch it.
#pragma once
#include "gemm_tc.cuh"

namespace p5 {

struct GemmPairCfg {
  static constexpr int BM = 128;  // rows per CTA: the pair covers 256
  static constexpr int BN = 256;  // columns of the pair's tile: each CTA stages 128 rows of B
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;        // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 384;  // 4 role warps + 8 epilogue warps
};

template <int EPI>
__global__ void __launch_bounds__(GemmPairCfg::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const GemmArgs args) {
  using C = GemmPairCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);  // [STAGES] own TMA landed
  uint64_t* empty_bar = full_bar + C::STAGES;   // [STAGES] pair MMAs done with the stage (multicast commit)
  uint64_t* pair_bar = empty_bar + C::STAGES;   // [STAGES] even CTA: the odd CTA's stage landed (relay)
  uint64_t* tfull_bar = pair_bar + C::STAGES;   // [2] accumulator complete (multicast commit)
  uint64_t* tempty_bar = tfull_bar + 2;         // [2] even CTA: accumulator drained by 16 epilogue warps
  uint64_t* done_bar = tempty_bar + 2;          // every pair MMA complete (multicast commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [2] skip

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool even = rank == 0;
  const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int kt_total = (args.K + C::BK - 1) / C::BK;
  const int n_units = args.tiles_m * args.tiles_n;  // 256 x 256 tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&pair_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 16);
    }
    mbar_init(done_bar, 1);
    flags[0] = 0;
    flags[2] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  cluster_sync();  // both CTAs' barriers exist before either side arrives remotely
  // a device-side wait already gave up in an earlier kernel: the even CTA decides for both, so the pair
  // skips (or runs) together
  if (even && threadIdx.x == 0 && args.status && *((volatile int*)args.status) != 0) {
    flags[2] = 1;
    st_cluster_u32(map_peer(smem_u32((const void*)&flags[2]), 1), 1u);
  }
  if (warp == 2) {
    tmem_alloc2(tmem_slot, C::TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool skip = flags[2] != 0;

  if (args.pdl) pdl_launch_dependents();

  auto decode = [&](int u, int& tm, int& tn) {
    const int per_group = args.group_m * args.tiles_n;
    const int group = u / per_group;
    const int first_m = group * args.group_m;
    const int gm = min(args.group_m, args.tiles_m - first_m);
    const int in_group = u % per_group;
    tm = first_m + in_group % gm;
    tn = in_group / gm;
  };

  if (skip) {
    // nothing issued: fall through to the common exit
  } else if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: this CTA's 128 rows of A and 128 rows of B per stage
      int it = 0;
      bool waited = !args.pdl;
      for (int u = cid; u < n_units && !flags[0]; u += nclusters) {
        int tm, tn;
        decode(u, tm, tn);
        const int arow = tm * 256 + (int)rank * 128, brow = tn * 256 + (int)rank * 128;
        for (int i = 0; i < kt_total; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.status, P5_ERR_WAIT_EMPTY)) {
            flags[0] = 1;
            break;
          }
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], i * C::BK, arow);
          tma_load_2d(sB + s * C::B_BYTES, &tma_b, &full_bar[s], i * C::BK, brow);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      if (even) {
        // ---------------- MMA issuer for the pair
        constexpr uint32_t idesc = mma_idesc_bf16(256, C::BN);
        int it = 0, j = 0;
        for (int u = cid; u < n_units && !flags[0]; u += nclusters, ++j) {
          const int acc = j & 1;
          const uint32_t aph = (uint32_t)(j >> 1) & 1u;
          if (!mbar_wait_cl(&tempty_bar[acc], aph ^ 1u, args.status, P5_ERR_WAIT_ACCUM)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * C::BN);
          for (int i = 0; i < kt_total; ++i, ++it) {
            const int s = it % C::STAGES;
            const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
            if (!mbar_wait(&full_bar[s], ph, args.status, P5_ERR_WAIT_FULL) ||
                !mbar_wait(&pair_bar[s], ph, args.status, P5_ERR_WAIT_FULL)) {
              flags[0] = 1;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES), b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
            for (int kk = 0; kk < C::BK / 16; ++kk)
              tc_mma2_f16(d_tmem, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32), idesc,
                          (i > 0 || kk > 0) ? 1u : 0u);
            tc_commit2_mc(&empty_bar[s], 3);  // frees the stage in both CTAs once these MMAs have read it
          }
          if (flags[0]) break;
          tc_commit2_mc(&tfull_bar[acc], 3);
        }
        tc_commit2_mc(done_bar, 3);  // lands once every MMA above has completed
      } else {
        // ---------------- relay: this CTA's stage landed -> the issuer's pair barrier
        const uint32_t pair0 = map_peer(smem_u32(pair_bar), 0);
        int it = 0;
        for (int u = cid; u < n_units && !flags[0]; u += nclusters) {
          for (int i = 0; i < kt_total; ++i, ++it) {
            const int s = it % C::STAGES;
            const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
            if (!mbar_wait(&full_bar[s], ph, args.status, P5_ERR_WAIT_FULL)) {
              flags[0] = 1;
              break;
            }
            mbar_arrive_cluster_relaxed(pair0 + (uint32_t)s * 8u);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue: this CTA's 128 rows of the pair's tile
    if (args.pdl) pdl_wait();
    const int sub = warp & 3;              // TMEM lanes [32*sub, 32*sub+32)
    const int c0 = ((warp - 4) >> 2) * (C::BN / 2);  // this warp's 128 columns
    const uint32_t lane_addr = (uint32_t)(sub * 32) << 16;
    const uint32_t tempty0 = map_peer(smem_u32(tempty_bar), 0);
    int j = 0;
    for (int u = cid; u < n_units; u += nclusters, ++j) {
      int tm, tn;
      decode(u, tm, tn);
      const int acc = j & 1;
      const uint32_t aph = (uint32_t)(j >> 1) & 1u;
      const bool ok = !flags[0] && mbar_wait(&tfull_bar[acc], aph, args.status, P5_ERR_WAIT_ACCUM);
      if (!ok) flags[0] = 1;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_addr + (uint32_t)(acc * C::BN);
      const int row = tm * 256 + (int)rank * 128 + sub * 32 + lane;
      const int col_base = tn * C::BN;
#pragma unroll 1
      for (int c = c0; c < c0 + C::BN / 2; c += 32) {
        uint32_t r[32];
        tmem_ld32(t_acc + (uint32_t)c, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = ok ? __uint_as_float(r[i]) : 0.f;
        if (ok) epi_chunk<EPI>(args, v, row, col_base + c);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (even)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_cluster(tempty0 + (uint32_t)acc * 8u);
      }
      if (!ok) break;
    }
  }

  // ---------------- exit: the issuer's last commit has landed in both CTAs, then both meet
  __syncthreads();
  if (!skip && threadIdx.x == 0) mbar_wait_cl(done_bar, 0, args.status, P5_ERR_WAIT_ACCUM);
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace p5

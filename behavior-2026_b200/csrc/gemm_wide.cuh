// gemm_wide.cuh — large GEMMs with 256x256 tiles per CTA (two M=128 tcgen05 MMAs sharing each B tile).
//
// Measured on B200: the mainloop of gemm_tc_kernel<256> (128x256 tiles) is bound by L2->shared-memory
// bandwidth — ~46 bytes per cycle per SM, which feeds 48 KB per 2.1 M MACs at about half the tensor
// rate.  A 256x256 tile loads 64 KB per 4.2 M MACs (A 256 rows + B 256 rows per 64-wide K block), 33 %
// fewer bytes per MAC.  The price: the two 128x256 fp32 accumulators fill all 512 TMEM columns, so
// there is no second accumulator to overlap the epilogue with the next tile's MMAs; eight epilogue
// warps (two per TMEM lane quarter, one per accumulator half) keep that drain short.  Three 64 KB
// stages of plain per-CTA TMA loads, same fused epilogues as gemm_tc_kernel (epi_row32), persistent CTAs
// walking the tiles in L2-sized groups of M tiles.  Used for K >= 4096, where the longer K loop
// amortises the unoverlapped drain.
#pragma once
#include "gemm_tc.cuh"

namespace p5 {

struct GemmWideCfg {
  static constexpr int BM = 256, BN = 256, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;  // two boxes of 128 rows
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 3;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
  static constexpr uint32_t TMEM_COLS = 512;
};

template <int EPI>
__global__ void __launch_bounds__(384, 1)
    gemm_wide_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const GemmArgs args) {
  using C = GemmWideCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;  // accumulators ready
  uint64_t* tempty_bar = tfull_bar + 1;         // accumulators drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] skip

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt_total = (args.K + C::BK - 1) / C::BK;
  const int n_units = args.tiles_m * args.tiles_n;

  if (threadIdx.x == 0) flags[1] = args.status ? *((volatile int*)args.status) : 0;
  __syncthreads();
  if (flags[1] != 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 8);  // one arrival per epilogue warp
    flags[0] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (args.pdl) pdl_launch_dependents();

  // unit -> (tm, tn): all N tiles of a group of M tiles whose A rows stay in L2
  auto decode = [&](int u, int& tm, int& tn) {
    const int per_group = args.group_m * args.tiles_n;
    const int group = u / per_group;
    const int first_m = group * args.group_m;
    const int gm = min(args.group_m, args.tiles_m - first_m);
    const int in_group = u % per_group;
    tm = first_m + in_group % gm;
    tn = in_group / gm;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      int it = 0;
      bool waited = !args.pdl;
      for (int u = blockIdx.x; u < n_units && !flags[0]; u += gridDim.x) {
        int tm, tn;
        decode(u, tm, tn);
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
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          tma_load_2d(st, &tma_a, &full_bar[s], i * C::BK, tm * C::BM);
          tma_load_2d(st + C::A_BYTES / 2, &tma_a, &full_bar[s], i * C::BK, tm * C::BM + 128);
          tma_load_2d(st + C::A_BYTES, &tma_b, &full_bar[s], i * C::BK, tn * C::BN);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: rows 0-127 -> TMEM columns 0-255, rows 128-255 -> 256-511
      constexpr uint32_t idesc = mma_idesc_bf16(128, C::BN);
      int it = 0, j = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++j) {
        if (!flags[0] && !mbar_wait(tempty_bar, ((uint32_t)j & 1u) ^ 1u, args.status, P5_ERR_WAIT_ACCUM)) flags[0] = 1;
        tc_fence_after();
        for (int i = 0; i < kt_total && !flags[0]; ++i, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(&full_bar[s], (uint32_t)(it / C::STAGES) & 1u, args.status, P5_ERR_WAIT_FULL)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES), b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {
            const uint64_t bd = sw128_kmajor_desc(b_addr + kk * 32);
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            tc_mma_f16(tmem_base, sw128_kmajor_desc(a_addr + kk * 32), bd, idesc, acc);
            tc_mma_f16(tmem_base + 256u, sw128_kmajor_desc(a_addr + C::A_BYTES / 2 + kk * 32), bd, idesc, acc);
          }
          tc_commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
        }
        tc_commit(tfull_bar);  // accumulators complete (or abandoned on abort)
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue: warp 4+4h+q drains rows [128h + 32q, +32) (TMEM lanes 32q.., columns 256h..)
    if (args.pdl) pdl_wait();
    const int half = (warp - 4) >> 2, sub = warp & 3;
    const uint32_t t_acc = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(half * 256);
    int j = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++j) {
      int tm, tn;
      decode(u, tm, tn);
      const bool ok = mbar_wait(tfull_bar, (uint32_t)j & 1u, args.status, P5_ERR_WAIT_ACCUM) && !flags[0];
      tc_fence_after();
      const int row = tm * C::BM + half * 128 + sub * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < C::BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(t_acc + (uint32_t)c, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (ok) epi_row32<EPI>(args, v, row, tn * C::BN + c);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace p5

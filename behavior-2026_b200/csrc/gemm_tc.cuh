// gemm_tc.cuh — tcgen05/TMEM GEMM for sm_100a:  D[M][N] = A[M][K] . B[N][K]^T, bf16 in, fp32 accumulate.
//
// One CTA computes one 128 x BN tile (optionally a K-slice of it, split-K).  Warp roles:
//   warp 0  TMA producer (one thread): STAGES-deep ring of (A, B) K-tiles of 64, 128-byte swizzle
//   warp 1  MMA issuer (one thread):   tcgen05.mma 128xBNx16, accumulator in TMEM (BN f32 columns)
//   warp 2  TMEM allocator
//   warps 4-7 epilogue: tcgen05.ld of their 32-lane TMEM sub-partition, fused epilogue, global stores
//
// The weights of every linear layer are stored [out][in] (K contiguous), so both operands are
// K-major.  Two orientations:
//   normal (swap = 0): A = activations [tokens][K], B = weights [features][K]; row = token, col = feature
//   swap   (swap = 1): A = weights, B = activations; row = feature, col = token.  Used when there are
//                      few tokens (the 50-token action expert): the 128-row MMA side walks the weights.
// Split-K partial tiles go to an fp32 workspace; the last CTA of a tile (ticket counter) sums the
// partials in split order, so results do not depend on CTA timing.
#pragma once
#include "common.cuh"

namespace p5 {

enum EpiKind : int {
  EPI_STORE = 0,  // out = R(v)
  EPI_GELU = 1,   // out = R(gelu(R(v)))
  EPI_RESID = 2,  // out = R(res + R(v))
  EPI_GATED = 3,  // out = R(res + R(R(v) * gate))          (adaRMS gated residual)
  EPI_GEGLU = 4,  // features interleaved (gate, up): out[f/2] = R(R(gelu(R(g))) * R(u))
  EPI_F32 = 5,    // out_f32 = v (no rounding)
};
// v = acc * out_scale + bias[f] + addend[(t % add_mod)][f]

struct GemmArgs {
  int M, N, K;           // GEMM extents (A rows, B rows, reduction)
  int swap;              // orientation (see above)
  int tiles_m, tiles_n;  // tile grid
  int group_m;           // tile-order grouping along M for L2 reuse
  int splits, kt_per_split;
  int epi;
  bf16* out;
  int ld_out;
  float* out_f32;
  int ld_out_f32;
  const bf16* bias;
  const bf16* res;
  int ld_res;
  const bf16* gate;
  int ld_gate, gate_div;
  float out_scale;
  const bf16* addend;
  int add_ld, add_mod;
  float* ws;
  int* counters;
  int* status;
  int pdl;  // kernel launched with programmatic stream serialization
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 128 ? 6 : 4);
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

// ---- epilogue value pipeline (one scalar) ----
__device__ __forceinline__ float epi_pre(const GemmArgs& a, float acc, int t, int f) {
  float v = acc;
  if (a.out_scale != 1.0f) v *= a.out_scale;
  if (a.bias) v += bf(a.bias[f]);
  if (a.addend) v += bf(a.addend[(size_t)(t % a.add_mod) * a.add_ld + f]);
  return v;
}
__device__ __forceinline__ float epi_final(const GemmArgs& a, float v, int t, int f) {
  switch (a.epi) {
    case EPI_GELU: return rbf(gelu_tanh(rbf(v)));
    case EPI_RESID: return rbf(bf(a.res[(size_t)t * a.ld_res + f]) + rbf(v));
    case EPI_GATED: {
      const float g = bf(a.gate[(size_t)(t / a.gate_div) * a.ld_gate + f]);
      return rbf(bf(a.res[(size_t)t * a.ld_res + f]) + rbf(rbf(v) * g));
    }
    default: return rbf(v);
  }
}

// Apply the epilogue to 32 accumulator values of one TMEM lane.
//   normal: row = token t, columns f0..f0+31 (features)
//   swap:   row = feature f, columns t0..t0+31 (tokens)
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, const float (&v)[32], int row, int col0, int lane) {
  if (!a.swap) {
    const int t = row, f0 = col0;
    if (t >= a.M) return;
    const int nf = min(32, a.N - f0);
    if (nf <= 0) return;
    if (a.epi == EPI_F32) {
      for (int i = 0; i < nf; ++i) a.out_f32[(size_t)t * a.ld_out_f32 + f0 + i] = epi_pre(a, v[i], t, f0 + i);
      return;
    }
    if (a.epi == EPI_GEGLU) {
      // columns (2j, 2j+1) = (gate_j, up_j)
      __align__(16) bf16 o[16];
      for (int j = 0; j < 16; ++j) {
        const float g = rbf(epi_pre(a, v[2 * j], t, f0 + 2 * j));
        const float u = rbf(epi_pre(a, v[2 * j + 1], t, f0 + 2 * j + 1));
        o[j] = tobf(rbf(gelu_tanh(g)) * u);
      }
      bf16* dst = a.out + (size_t)t * a.ld_out + f0 / 2;
      if (nf == 32) {
        reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<const uint4*>(o)[0];
        reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<const uint4*>(o)[1];
      } else {
        for (int j = 0; j < nf / 2; ++j) dst[j] = o[j];
      }
      return;
    }
    __align__(16) bf16 o[32];
    for (int i = 0; i < 32; ++i) o[i] = tobf(i < nf ? epi_final(a, epi_pre(a, v[i], t, f0 + i), t, f0 + i) : 0.f);
    bf16* dst = a.out + (size_t)t * a.ld_out + f0;
    if (nf == 32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(dst)[q] = reinterpret_cast<const uint4*>(o)[q];
    } else {
      for (int i = 0; i < nf; ++i) dst[i] = o[i];
    }
  } else {
    const int f = row, t0 = col0;
    const bool fok = f < a.M;
    if (a.epi == EPI_GEGLU) {
      // rows (2j, 2j+1) = (gate_j, up_j): partner lives in the neighbouring lane
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int t = t0 + i;
        float mine = fok ? rbf(epi_pre(a, v[i], t, f)) : 0.f;
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        if (fok && (f & 1) == 0 && t < a.N) a.out[(size_t)t * a.ld_out + f / 2] = tobf(rbf(gelu_tanh(mine)) * other);
      }
      return;
    }
    if (!fok) return;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
      const int t = t0 + i;
      if (t >= a.N) break;
      if (a.epi == EPI_F32) {
        a.out_f32[(size_t)t * a.ld_out_f32 + f] = epi_pre(a, v[i], t, f);
      } else {
        a.out[(size_t)t * a.ld_out + f] = tobf(epi_final(a, epi_pre(a, v[i], t, f), t, f));
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(256, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const GemmArgs args) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* accum_bar = empty_bar + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last split, [2] skip

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile coordinates (grouped along M so consecutive CTAs share B tiles in L2)
  const int tile = blockIdx.x;
  const int per_group = args.group_m * args.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * args.group_m;
  const int gm = min(args.group_m, args.tiles_m - first_m);
  const int in_group = tile % per_group;
  const int tm = first_m + in_group % gm;
  const int tn = in_group / gm;
  const int m0 = tm * C::BM, n0 = tn * BN;
  const int split = blockIdx.y;
  const int kt_total = (args.K + C::BK - 1) / C::BK;
  const int kt0 = split * args.kt_per_split;
  const int kt1 = min(kt_total, kt0 + args.kt_per_split);
  const int nkt = max(0, kt1 - kt0);

  // a device-side wait already gave up in an earlier kernel: skip the work (uniformly for the CTA)
  if (threadIdx.x == 0) flags[2] = args.status ? *((volatile int*)args.status) : 0;
  __syncthreads();
  if (flags[2] != 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accum_bar, 1);
    flags[0] = 0;
    flags[1] = 0;
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

  if (warp == 0) {
    if (lane == 0) {
    // ---------------- producer
    // In swap orientation A holds weights, which never depend on the previous kernel, so the
    // first stages of A are requested before waiting for the predecessor grid.
    const int pre = args.swap && args.pdl ? min(nkt, C::STAGES) : 0;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full_bar[i], C::STAGE_BYTES);
      tma_load_2d(sA + i * C::A_BYTES, &tma_a, &full_bar[i], (kt0 + i) * C::BK, m0);
    }
    if (args.pdl) pdl_wait();
    for (int i = 0; i < nkt; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
      if (i >= pre) {
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.status, P5_ERR_WAIT_EMPTY)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
        tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], (kt0 + i) * C::BK, m0);
      }
      tma_load_2d(sB + s * C::B_BYTES, &tma_b, &full_bar[s], (kt0 + i) * C::BK, n0);
    }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
    // ---------------- MMA issuer
    if (args.pdl) pdl_wait();
    constexpr uint32_t idesc = mma_idesc_bf16(C::BM, BN);
    for (int i = 0; i < nkt; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
      if (flags[0] || !mbar_wait(&full_bar[s], ph, args.status, P5_ERR_WAIT_FULL)) {
        flags[0] = 1;
        break;
      }
      tc_fence_after();
      const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES), b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < C::BK / 16; ++kk) {
        tc_mma_f16(tmem_base, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32), idesc,
                   (i > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
    }
    tc_commit(accum_bar);  // accumulator complete
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue
    if (args.pdl) pdl_wait();
    const int sub = warp & 3;  // TMEM lanes [32*sub, 32*sub+32)
    const int row = m0 + sub * 32 + lane;
    const bool ok = mbar_wait(accum_bar, 0, args.status, P5_ERR_WAIT_ACCUM) && nkt > 0;
    tc_fence_after();
    const int ntid = 128;
    if (args.splits == 1) {
      if (ok) {
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)c, r);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          epilogue_chunk(args, v, row, n0 + c, lane);
        }
      }
    } else {
      // split-K: write the partial tile, take a ticket, the last split reduces in split order
      const int tile_id = tm * args.tiles_n + tn;
      const size_t tile_elems = (size_t)C::BM * BN;
      float* mine = args.ws + ((size_t)split * args.tiles_m * args.tiles_n + tile_id) * tile_elems;
      const int lrow = sub * 32 + lane;
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        if (ok) {
          tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)c, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        float4* dst = reinterpret_cast<float4*>(mine + (size_t)lrow * BN + c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                               __uint_as_float(r[4 * q + 3]));
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(ntid));
      if (threadIdx.x == 128) {
        const int prev = atomicAdd(&args.counters[tile_id], 1);
        flags[1] = (prev == args.splits - 1) ? 1 : 0;
        if (prev == args.splits - 1) args.counters[tile_id] = 0;  // re-arm for the next launch
      }
      asm volatile("bar.sync 1, %0;" ::"r"(ntid));
      if (flags[1]) {
        __threadfence();
        for (int c = 0; c < BN; c += 32) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
          for (int s = 0; s < args.splits; ++s) {
            const float4* src = reinterpret_cast<const float4*>(
                args.ws + ((size_t)s * args.tiles_m * args.tiles_n + tile_id) * tile_elems + (size_t)lrow * BN + c);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 p = __ldcg(src + q);
              v[4 * q] += p.x;
              v[4 * q + 1] += p.y;
              v[4 * q + 2] += p.z;
              v[4 * q + 3] += p.w;
            }
          }
          epilogue_chunk(args, v, row, n0 + c, lane);
        }
      }
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

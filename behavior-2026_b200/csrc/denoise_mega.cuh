// denoise_mega.cuh — the whole flow-matching denoise of one sample as one persistent kernel.
//
// One CTA per SM (cooperative launch, so every CTA is resident) walks
//   for each step:  action_in | 18 x [ QKV+RoPE | attention | split merge | O+gate | GU+GeGLU | down+gate ]
//                   | final adaRMSNorm + action_out + Euler
// with a grid-wide barrier between phases (110 per step).  What the per-kernel path pays per launch
// (launch latency, prologue, a full drain before the next kernel may read) becomes one barrier, and
// the weights of a CTA's next GEMM phase are fetched by TMA into shared memory while it is still in
// the current phase or waiting at the barrier, so the 34.6 MB of weights per layer stream from HBM
// behind the latency chain instead of on it.
//
// GEMM phases (action tokens T <= 64 on the N side, 128 weight rows per tile on the M side, tcgen05
// with the accumulator in TMEM): a unit = (row tile, K split); each CTA computes one unit's partial
// tile, the S CTAs of a tile meet at a counter in global memory, and each reduces 1/S of the tile's
// outputs over the S partials in split order (deterministic) and applies the phase's epilogue:
//   QKV  F=2560 K=1024 S=6   rows of each 256-wide head interleaved (2j = dim j, 2j+1 = dim j+128), so a
//                            tile holds both halves of its RoPE pairs: RoPE, q*1/16 and K/V writes in the reduce
//   O    F=1024 K=2048 S=16  x += R(R(acc) * gate1)
//   GU   F=8192 K=1024 S=2   interleaved gate/up rows: act = R(R(gelu(R(g))) * R(u))
//   DN   F=1024 K=4096 S=16  x += R(R(acc) * gate2)
// The adaRMSNorm in front of QKV and GU is applied while building the B operand: each CTA computes
// the 1/rms of every token from x and normalises only its own K range into swizzled shared memory.
// Attention is attn_tc_body (tcgen05, split-KV) on 4 x splits CTAs, merged by all CTAs.
// Rounding points and formulas are those of the per-kernel path (rmsnorm_kernel, rope_qkv_kernel,
// the GEMM epilogues, action_in_kernel, action_out_euler_kernel).
#pragma once
#include "attention_tc.cuh"
#include "pi05_model.h"

namespace p5 {

enum { MG_QKV = 0, MG_O = 1, MG_GU = 2, MG_DN = 3 };
__host__ __device__ constexpr int mg_F(int p) { return p == MG_QKV ? P5_QKV : p == MG_GU ? 2 * P5_EXP_MLP : P5_EXP_W; }
__host__ __device__ constexpr int mg_K(int p) {
  return p == MG_QKV ? P5_EXP_W : p == MG_O ? P5_QDIM : p == MG_GU ? P5_EXP_W : P5_EXP_MLP;
}
__host__ __device__ constexpr int mg_kbps(int p) { return p == MG_QKV ? 3 : p == MG_O ? 2 : p == MG_GU ? 8 : 4; }
__host__ __device__ constexpr int mg_S(int p) { return (mg_K(p) / 64 + mg_kbps(p) - 1) / mg_kbps(p); }
__host__ __device__ constexpr int mg_tiles(int p) { return mg_F(p) / 128; }
__host__ __device__ constexpr int mg_units(int p) { return mg_tiles(p) * mg_S(p); }
__host__ __device__ constexpr int mg_ctr_off(int p) {  // tile counters follow the grid counter
  return 1 + (p > 0 ? mg_tiles(0) : 0) + (p > 1 ? mg_tiles(1) : 0) + (p > 2 ? mg_tiles(2) : 0);
}
constexpr int MG_NCTR = 1 + 20 + 8 + 64 + 8;

struct MegaCfg {
  static constexpr int THREADS = 384;
  static constexpr int A_KB = 16384;  // one 64-wide K block of 128 weight rows
  static constexpr int B_OFF = 8 * A_KB, B_KB = 8192;  // one K block of 64 token rows
  static constexpr int MISC_OFF = AttnTcCfg::BAR_OFF + 256;  // past attn_tc_body's own barriers
  static constexpr int SMEM = 1024 + MISC_OFF + 512;
  static constexpr int NMAPS_LAYER = 6;  // qkv (row-permuted), o, gu, down, K cache, V cache
};
static_assert(MegaCfg::B_OFF + 8 * MegaCfg::B_KB <= AttnTcCfg::BAR_OFF, "GEMM buffers overlap the misc area");

struct MegaArgs {
  bf16* x;        // [T][1024] residual stream
  float* xt;      // [T][32] action state (fp32)
  bf16* qkv;      // [T][2560]: q (after RoPE and 1/16) in columns 0..2047
  bf16* ek;       // [T][256] action-token K after RoPE
  bf16* ev;       // [T][256] action-token V
  bf16* eo;       // [T][2048] attention output
  bf16* act;      // [T][4096] GeGLU output
  float* ws;      // GEMM partial tiles [unit][128][64]
  float* attn_o;  // attention split partials
  float* attn_ml;
  int attn_half;  // attention split partials as fp16 O / l (as the per-kernel path stores them)
  unsigned* ctr;  // [0] grid barrier, then per-tile counters; zero at launch
  int* status;
  const bf16* mods;  // [steps][NM][3][1024] adaRMS scale, shift, gate
  const bf16 *ain_w, *ain_b, *aout_w, *aout_b;
  const float *cos_t, *sin_t;
  const CUtensorMap* maps;  // [L][6] per layer, then q, ek, ev, eo, act
  int T, P, L, steps, NM;
  float dtb;
  int attn_splits, attn_tps;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Arrive on *ctr and wait until it reaches `target` (thread 0 spins, bounded).  False when the wait
// gave up or a device-side error is already recorded; the caller then leaves the kernel.
__device__ __forceinline__ bool mg_counter_sync(unsigned* ctr, unsigned target, int* status, volatile int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(ctr, 1u);
    const unsigned long long t0 = clock64();
    while (ld_acquire_u32(ctr) < target) {
      if (*(volatile int*)status != 0) {
        ok = 0;
        break;
      }
      if ((unsigned long long)clock64() - t0 > P5_WAIT_CYCLES) {
        record_error(status, P5_ERR_WAIT_GRID);
        ok = 0;
        break;
      }
    }
    if (ok && *(volatile int*)status != 0) ok = 0;
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// Per-CTA state of the persistent kernel (identical in every thread of the CTA).
struct MegaCtx {
  const MegaArgs& a;
  uint8_t* smem;
  uint8_t* sA;
  uint8_t* sB;
  uint64_t* w_full;  // this CTA's next weight slice landed
  uint64_t* b_full;  // B operand landed (TMA phases)
  uint64_t* mma_done;
  volatile int* flags;
  float* inv_rms;  // [64]
  uint32_t tmem_base;
  int tid, warp, lane, G, cta, attn_first;
  uint32_t w_uses = 0, b_uses = 0, m_uses = 0;
  bool w_pending = false;
  unsigned grid_target = 0;
  __device__ MegaCtx(const MegaArgs& args) : a(args) {}

  __device__ bool grid_sync() {
    grid_target += (unsigned)G;
    return mg_counter_sync(&a.ctr[0], grid_target, a.status, flags);
  }

  // weights of this CTA's unit in GEMM phase P of layer l -> shared memory (one thread issues)
  template <int P>
  __device__ void prefetch(int l) {
    if (cta >= mg_units(P)) return;
    constexpr int S = mg_S(P);
    const int tile = cta / S, split = cta % S;
    const int kb0 = split * mg_kbps(P), nkb = min(mg_kbps(P), mg_K(P) / 64 - kb0);
    if (tid == 0) {
      const CUtensorMap* m = a.maps + l * MegaCfg::NMAPS_LAYER + P;
      mbar_arrive_expect_tx(w_full, (uint32_t)(nkb * MegaCfg::A_KB));
      for (int kb = 0; kb < nkb; ++kb) tma_load_2d(sA + kb * MegaCfg::A_KB, m, w_full, (kb0 + kb) * 64, tile * 128);
    }
    w_pending = true;
  }

  // 1/rms of every token row of x (adaRMSNorm statistics): warp w takes rows w, w+12, ...; all of a
  // warp's loads are issued before the first add
  __device__ void row_stats() {
    constexpr int D = P5_EXP_W, NWARP = MegaCfg::THREADS / 32, RPW = (64 + NWARP - 1) / NWARP;  // 6
    uint4 u[RPW][4];  // all 24 loads of a lane in flight together
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int t = warp + r * NWARP;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        u[r][q] = t < a.T ? __ldcg(reinterpret_cast<const uint4*>(a.x + (long)t * D + q * 256 + lane * 8))
                          : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w[4] = {u[r][q].x, u[r][q].y, u[r][q].z, u[r][q].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf2(w[k]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const int t = warp + r * NWARP;
      if (lane == 0 && t < 64) inv_rms[t] = 1.0f / sqrtf(ss / (float)D + 1e-6f);
    }
    __syncthreads();
  }

  // adaRMSNorm(x) (scale = mod, shift = mod + D) for K blocks [kb0, kb0+NKB) -> B operand tiles
  template <int NKB>
  __device__ void build_norm_b(int kb0, int nkb, const bf16* mod) {
    constexpr int D = P5_EXP_W, PER_T = NKB * 8, ITEMS = 64 * PER_T;
    constexpr int IPT = (ITEMS + MegaCfg::THREADS - 1) / MegaCfg::THREADS, BATCH = 4;
#pragma unroll 1
    for (int b0 = 0; b0 < IPT; b0 += BATCH) {
      uint4 xv[BATCH], sv[BATCH], hv[BATCH];  // a batch's loads are all in flight before the math
#pragma unroll
      for (int it = 0; it < BATCH; ++it) {
        const int i = tid + (b0 + it) * MegaCfg::THREADS;
        const int t = i / PER_T, rem = i % PER_T, kb = rem >> 3, c = rem & 7;
        const int k = (kb0 + kb) * 64 + c * 8;
        const bool ok = b0 + it < IPT && i < ITEMS && kb < nkb && t < a.T;
        xv[it] = ok ? __ldcg(reinterpret_cast<const uint4*>(a.x + (long)t * D + k)) : make_uint4(0u, 0u, 0u, 0u);
        sv[it] = ok ? *reinterpret_cast<const uint4*>(mod + k) : make_uint4(0u, 0u, 0u, 0u);
        hv[it] = ok ? *reinterpret_cast<const uint4*>(mod + D + k) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int it = 0; it < BATCH; ++it) {
        const int i = tid + (b0 + it) * MegaCfg::THREADS;
        const int t = i / PER_T, rem = i % PER_T, kb = rem >> 3, c = rem & 7;
        if (b0 + it >= IPT || i >= ITEMS || kb >= nkb) continue;
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (t < a.T) {
          const float inv = inv_rms[t];
          const uint32_t w[4] = {xv[it].x, xv[it].y, xv[it].z, xv[it].w},
                         ws[4] = {sv[it].x, sv[it].y, sv[it].z, sv[it].w}, wh[4] = {hv[it].x, hv[it].y, hv[it].z, hv[it].w};
          uint32_t r[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf2(w[q]), s2 = unpack_bf2(ws[q]), h2 = unpack_bf2(wh[q]);
            r[q] = pack_bf2(f.x * inv * rbf(1.0f + s2.x) + h2.x, f.y * inv * rbf(1.0f + s2.y) + h2.y);
          }
          o = make_uint4(r[0], r[1], r[2], r[3]);
        }
        *reinterpret_cast<uint4*>(sB + kb * MegaCfg::B_KB + t * 128 + ((c ^ (t & 7)) << 4)) = o;
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
  }

  // Sum over the S partial tiles (in split order) of rows r0, r1 at token t.
  template <int S>
  __device__ __forceinline__ void psum2(const float* part, int r0, int r1, int t, float& v0, float& v1) {
    float p0[S], p1[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
      p0[s] = __ldcg(part + ((size_t)s * 128 + r0) * 64 + t);
      p1[s] = __ldcg(part + ((size_t)s * 128 + r1) * 64 + t);
    }
    v0 = 0.f;
    v1 = 0.f;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      v0 += p0[s];
      v1 += p1[s];
    }
  }

  // One GEMM phase for this CTA's unit.  False if a wait gave up.
  template <int P>
  __device__ bool gemm_phase(int l, int use, const bf16* mod) {
    using C = MegaCfg;
    constexpr int D = P5_EXP_W, S = mg_S(P), KBPS = mg_kbps(P);
    constexpr bool TMA_B = (P == MG_O || P == MG_DN);
    const bool has = cta < mg_units(P);
    const int tile = cta / S, split = cta % S;
    const int kb0 = split * KBPS, nkb = has ? min(KBPS, mg_K(P) / 64 - kb0) : 0;
    if (has) {
      // ---- B operand: 64 token rows x this unit's K range, 128-byte swizzled, K-major
      if (TMA_B) {
        if (tid == 0) {
          const CUtensorMap* m = a.maps + a.L * C::NMAPS_LAYER + (P == MG_O ? 3 : 4);
          mbar_arrive_expect_tx(b_full, (uint32_t)(nkb * C::B_KB));
          for (int kb = 0; kb < nkb; ++kb) tma_load_2d(sB + kb * C::B_KB, m, b_full, (kb0 + kb) * 64, 0);
        }
      } else {
        row_stats();
        build_norm_b<KBPS>(kb0, nkb, mod);
      }
      // ---- MMA: D[128 weight rows][64 tokens] in TMEM columns 0..63
      if (warp == 1 && lane == 0) {
        bool ok = mbar_wait(w_full, w_uses & 1u, a.status, P5_ERR_WAIT_FULL);
        if (TMA_B) ok = ok && mbar_wait(b_full, b_uses & 1u, a.status, P5_ERR_WAIT_FULL);
        tc_fence_after();
        if (ok) {
          constexpr uint32_t idesc = mma_idesc_bf16(128, 64);
          const uint32_t aa = smem_u32(sA), ba = smem_u32(sB);
          for (int kb = 0; kb < nkb; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f16(tmem_base, sw128_kmajor_desc(aa + kb * C::A_KB + kk * 32),
                         sw128_kmajor_desc(ba + kb * C::B_KB + kk * 32), idesc, (kb | kk) ? 1u : 0u);
        }
        tc_commit(mma_done);
      }
      ++w_uses;
      w_pending = false;
      if (TMA_B) ++b_uses;
      // ---- partial tile -> global workspace [unit][row][token]
      if (warp >= 4 && warp < 8) {
        const int sub = warp - 4, row = sub * 32 + lane;
        const bool ok = mbar_wait(mma_done, m_uses & 1u, a.status, P5_ERR_WAIT_ACCUM);
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16), r0);
        tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + 32u, r1);
        tmem_wait_ld();
        float4* dst = reinterpret_cast<float4*>(a.ws + ((size_t)cta * 128 + row) * 64);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          dst[q] = ok ? make_float4(__uint_as_float(r0[4 * q]), __uint_as_float(r0[4 * q + 1]),
                                    __uint_as_float(r0[4 * q + 2]), __uint_as_float(r0[4 * q + 3]))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
          dst[8 + q] = ok ? make_float4(__uint_as_float(r1[4 * q]), __uint_as_float(r1[4 * q + 1]),
                                        __uint_as_float(r1[4 * q + 2]), __uint_as_float(r1[4 * q + 3]))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      ++m_uses;
      tc_fence_before();
      __syncthreads();  // warps 4-7 saw every MMA complete: shared memory is free again
    }
    // ---- the next GEMM phase's weights (O waits until after attention on the attention CTAs)
    if (P == MG_QKV && cta < attn_first) prefetch<MG_O>(l);
    if (P == MG_O) prefetch<MG_GU>(l);
    if (P == MG_GU) prefetch<MG_DN>(l);
    if (P == MG_DN && !(l == a.L - 1 && use == a.steps * a.L - 1)) prefetch<MG_QKV>((l + 1) % a.L);
    if (!has) return true;
    // ---- the S units of this tile meet; each reduces its share of the tile
    if (!mg_counter_sync(&a.ctr[mg_ctr_off(P) + tile], (unsigned)((use + 1) * S), a.status, flags)) return false;
    const float* part = a.ws + (size_t)tile * S * 128 * 64;
    const int T = a.T;
    if (P == MG_QKV) {
      // rows (2r, 2r+1) of the interleaved tile = head dims (j, j+128), j = (tile % 2) * 64 + r
      const int n = 64 * T, i0 = split * n / S, i1 = (split + 1) * n / S;
      const int hb = tile >> 1, j0 = (tile & 1) * 64;
      for (int i = i0 + tid; i < i1; i += C::THREADS) {
        const int r = i / T, t = i % T, j = j0 + r;
        float v0, v1;
        psum2<S>(part, 2 * r, 2 * r + 1, t, v0, v1);
        const float x1 = rbf(v0), x2 = rbf(v1);
        if (hb == 9) {
          a.ev[(long)t * P5_HD + j] = tobf(x1);
          a.ev[(long)t * P5_HD + j + 128] = tobf(x2);
          continue;
        }
        const int pos = a.P + t;
        const float cs = a.cos_t[(long)pos * 128 + j], sn = a.sin_t[(long)pos * 128 + j];
        const float ra = rbf(x1 * cs - x2 * sn);
        const float rc = rbf(x2 * cs + x1 * sn);
        if (hb == 8) {
          a.ek[(long)t * P5_HD + j] = tobf(ra);
          a.ek[(long)t * P5_HD + j + 128] = tobf(rc);
        } else {
          a.qkv[(long)t * P5_QKV + hb * P5_HD + j] = tobf(ra * 0.0625f);
          a.qkv[(long)t * P5_QKV + hb * P5_HD + j + 128] = tobf(rc * 0.0625f);
        }
      }
    } else if (P == MG_GU) {
      // rows (2jj, 2jj+1) = (gate, up) of GeGLU output column tile*64 + jj
      const int n = 64 * T, i0 = split * n / S, i1 = (split + 1) * n / S;
      for (int i = i0 + tid; i < i1; i += C::THREADS) {
        const int jj = i / T, t = i % T;
        float g, u;
        psum2<S>(part, 2 * jj, 2 * jj + 1, t, g, u);
        a.act[(long)t * P5_EXP_MLP + tile * 64 + jj] = tobf(rbf(gelu_tanh(rbf(g))) * rbf(u));
      }
    } else {
      // x += R(R(acc) * gate); two rows per item
      const bf16* gate = mod + 2 * D;
      const int n = 64 * T, i0 = split * n / S, i1 = (split + 1) * n / S;
      for (int i = i0 + tid; i < i1; i += C::THREADS) {
        const int r = i / T, t = i % T;
        float v0, v1;
        psum2<S>(part, r, r + 64, t, v0, v1);
        const int f0 = tile * 128 + r, f1 = f0 + 64;
        bf16* x0 = a.x + (long)t * D + f0;
        bf16* x1 = a.x + (long)t * D + f1;
        *x0 = tobf(bf(*x0) + rbf(rbf(v0) * bf(gate[f0])));
        *x1 = tobf(bf(*x1) + rbf(rbf(v1) * bf(gate[f1])));
      }
    }
    return true;
  }
};

__global__ void __launch_bounds__(MegaCfg::THREADS, 1) denoise_mega_kernel(const MegaArgs a) {
  using C = MegaCfg;
  constexpr int D = P5_EXP_W;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  MegaCtx c(a);
  c.smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  c.sA = c.smem;
  c.sB = c.smem + C::B_OFF;
  c.w_full = reinterpret_cast<uint64_t*>(c.smem + C::MISC_OFF);
  c.b_full = c.w_full + 1;
  c.mma_done = c.w_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(c.w_full + 3);
  c.flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] sync result, [1] start status
  c.inv_rms = reinterpret_cast<float*>(c.smem + C::MISC_OFF + 64);
  c.tid = threadIdx.x;
  c.warp = threadIdx.x >> 5;
  c.lane = threadIdx.x & 31;
  c.G = gridDim.x;
  c.cta = blockIdx.x;
  const int tid = c.tid, warp = c.warp, lane = c.lane, G = c.G, cta = c.cta, T = a.T;

  if (tid == 0) c.flags[1] = *((volatile int*)a.status);
  __syncthreads();
  if (c.flags[1] != 0) return;

  if (tid == 0) {
    mbar_init(c.w_full, 1);
    mbar_init(c.b_full, 1);
    mbar_init(c.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, AttnTcCfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem_base = *tmem_slot;
  const int n_rb = (T * 8 + 127) / 128;
  c.attn_first = G - n_rb * a.attn_splits;  // the last CTAs run attention
  const CUtensorMap* gmaps = a.maps + a.L * C::NMAPS_LAYER;

  bool alive = true;
  if (a.steps > 0 && a.L > 0) c.prefetch<MG_QKV>(0);
  for (int s = 0; s < a.steps && alive; ++s) {
    const bf16* mrow = a.mods + (size_t)s * a.NM * 3 * D;
    // ---- action_in: x = W_in xt + b (vector loads, k in order)
    for (long idx = (long)cta * C::THREADS + tid; idx < (long)T * D; idx += (long)G * C::THREADS) {
      const int t = (int)(idx / D), o = (int)(idx % D);
      const float4* xv = reinterpret_cast<const float4*>(a.xt + (long)t * P5_ACT_D);
      const uint4* wv = reinterpret_cast<const uint4*>(a.ain_w + (long)o * P5_ACT_D);
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < P5_ACT_D / 8; ++q) {
        float wf[8];
        unpack8(wv[q], wf);
        const float4 x0 = xv[2 * q], x1 = xv[2 * q + 1];
        acc += x0.x * wf[0];
        acc += x0.y * wf[1];
        acc += x0.z * wf[2];
        acc += x0.w * wf[3];
        acc += x1.x * wf[4];
        acc += x1.y * wf[5];
        acc += x1.z * wf[6];
        acc += x1.w * wf[7];
      }
      a.x[idx] = tobf(acc + bf(a.ain_b[o]));
    }
    if (!c.grid_sync()) {
      alive = false;
      break;
    }
    for (int l = 0; l < a.L; ++l) {
      const int use = s * a.L + l;
      const bf16* m1 = mrow + (size_t)(2 * l) * 3 * D;
      const bf16* m2 = mrow + (size_t)(2 * l + 1) * 3 * D;
      // ---- q/k/v projection + RoPE
      if (!c.gemm_phase<MG_QKV>(l, use, m1) || !c.grid_sync()) {
        alive = false;
        break;
      }
      // ---- attention over [prefix cache || action tokens], split-KV partials
      AttnArgs at = {};
      at.q = a.qkv;
      at.ldq = P5_QKV;
      at.q_bstride = (long)T * P5_QKV;
      at.out = a.eo;
      at.ldo = P5_QDIM;
      at.o_bstride = (long)T * P5_QDIM;
      at.len1 = a.P;
      at.len2 = T;
      at.T = T;
      at.G = P5_NH;
      at.qdiv = 1.0f;
      at.splits = a.attn_splits;
      at.keys_per_split = a.attn_tps * AttnTcCfg::KT;
      at.ws_o = a.attn_o;
      at.ws_ml = a.attn_ml;
      at.ws_half = a.attn_half;
      if (cta >= c.attn_first) {
        const int u = cta - c.attn_first;
        const CUtensorMap* lm = a.maps + l * C::NMAPS_LAYER;
        attn_tc_body(at, gmaps + 0, lm + 4, lm + 5, gmaps + 1, gmaps + 2, a.status, c.smem, c.tmem_base,
                     u / a.attn_splits, u % a.attn_splits);
        c.prefetch<MG_O>(l);
      }
      if (!c.grid_sync()) {
        alive = false;
        break;
      }
      // ---- merge the key splits -> eo
      for (long idx = (long)cta * C::THREADS + tid; idx < (long)T * 8 * (P5_HD / 2); idx += (long)G * C::THREADS)
        attn_combine_item<P5_HD>(at, idx);
      if (!c.grid_sync()) {
        alive = false;
        break;
      }
      // ---- O projection + gated residual, GU + GeGLU, down + gated residual
      if (!c.gemm_phase<MG_O>(l, use, m1) || !c.grid_sync() || !c.gemm_phase<MG_GU>(l, use, m2) || !c.grid_sync() ||
          !c.gemm_phase<MG_DN>(l, use, m2) || !c.grid_sync()) {
        alive = false;
        break;
      }
    }
    if (!alive) break;
    // ---- final adaRMSNorm + action_out + Euler: warp per (token, action dim); the warp normalises
    // the token's row itself (same rounding as rmsnorm_kernel + action_out_euler_kernel)
    {
      const bf16* mf = mrow + (size_t)(a.NM - 1) * 3 * D;
      const int gw = cta * (C::THREADS / 32) + warp, nw = G * (C::THREADS / 32);
      for (int w = gw; w < T * P5_ACT_D; w += nw) {
        const int t = w / P5_ACT_D, j = w % P5_ACT_D;
        const bf16* xr = a.x + (long)t * D;
        const bf16* wr = a.aout_w + (long)j * D;
        uint4 xu[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) xu[q] = __ldcg(reinterpret_cast<const uint4*>(xr + q * 256 + lane * 8));
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t wv[4] = {xu[q].x, xu[q].y, xu[q].z, xu[q].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf2(wv[k]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / (float)D + 1e-6f);
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = q * 256 + lane * 8;
          const uint4 cu = *reinterpret_cast<const uint4*>(wr + k);
          const uint4 us = *reinterpret_cast<const uint4*>(mf + k), uh = *reinterpret_cast<const uint4*>(mf + D + k);
          const uint32_t xa[4] = {xu[q].x, xu[q].y, xu[q].z, xu[q].w}, cc[4] = {cu.x, cu.y, cu.z, cu.w},
                         sa[4] = {us.x, us.y, us.z, us.w}, ha[4] = {uh.x, uh.y, uh.z, uh.w};
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2) {
            const float2 f = unpack_bf2(xa[k2]), s2 = unpack_bf2(sa[k2]), h2 = unpack_bf2(ha[k2]), g = unpack_bf2(cc[k2]);
            const float hx = rbf(f.x * inv * rbf(1.0f + s2.x) + h2.x), hy = rbf(f.y * inv * rbf(1.0f + s2.y) + h2.y);
            acc += hx * g.x + hy * g.y;
          }
        }
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
          const float v = rbf(acc + bf(a.aout_b[j]));
          a.xt[(long)t * P5_ACT_D + j] += rbf(a.dtb * v);
        }
      }
    }
    if (!c.grid_sync()) {
      alive = false;
      break;
    }
  }

  // a weight prefetch still in flight must land before this CTA's shared memory goes away
  if (c.w_pending && warp == 0 && lane == 0) mbar_wait(c.w_full, c.w_uses & 1u, a.status, P5_ERR_WAIT_FULL);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(c.tmem_base, AttnTcCfg::TMEM_COLS);
  }
}

// Row interleaving of a q/k/v weight [2560][K] for the fused-RoPE projections: within each 256-row
// head block, row 2j takes head dim j and row 2j+1 head dim j+128.
__global__ void interleave_qkv_rows_kernel(const bf16* src, bf16* dst, int K) {
  const int drow = blockIdx.x;  // 0..2559
  const int hb = drow >> 8, w = drow & 255;
  const int srow = hb * 256 + (w >> 1) + (w & 1) * 128;
  const uint4* s = reinterpret_cast<const uint4*>(src + (long)srow * K);
  uint4* d = reinterpret_cast<uint4*>(dst + (long)drow * K);
  for (int i = threadIdx.x; i < K / 8; i += blockDim.x) d[i] = s[i];
}

}  // namespace p5

// gemm_tc.cuh — tcgen05/TMEM GEMM for sm_100a:  D[M][N] = A[M][K] . B[N][K]^T, bf16 in, fp32 accumulate.
//
// Persistent: the grid has at most one CTA per SM and each CTA walks work units (tile, K-split)
// u = blockIdx.x, blockIdx.x + gridDim.x, ...  Warp roles:
//   warp 0  TMA producer (lane 0): STAGES-deep ring of (A, B) K-tiles of 64, 128-byte swizzle;
//           the ring runs on across units, so the next tile's loads start while this one computes
//   warp 1  MMA issuer (lane 0): tcgen05.mma 128xBNx16 into one of two TMEM accumulators
//   warp 2  TMEM allocator (2 x BN f32 columns)
//   warps 4-7 epilogue: tcgen05.ld of their 32-lane TMEM sub-partition, fused epilogue, stores.
//           The accumulator is handed back as soon as it is read, so the epilogue of unit j
//           overlaps the MMAs of unit j+1.
//
// Every linear layer stores its weights [out][in] (K contiguous): both operands are K-major.
//   normal (swap = 0): A = activations [tokens][K], B = weights [features][K]; row = token, col = feature
//   swap   (swap = 1): A = weights, B = activations; row = feature, col = token.  Used for few tokens
//                      (the 50-token action expert): the 128-row MMA side walks the weights.
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
  // small-N epilogues of the LoRA path (normal orientation, BN <= 48)
  EPI_STORE_T = 6,    // x = R(v*out_scale): out[t][f] = x and out_t[f][t] = x (transposed copy)
  EPI_LORA_GRAD = 7,  // fp32 gradient accumulate: D[m][c] with adapter c/16 (see GemmArgs lg_*)
  // q/k/v projection with RoPE fused (normal orientation, or swap orientation through the cluster
  // reduce): the weight rows of each 256-wide head are interleaved (row 2j = dim j, row 2j+1 = dim
  // j+128), see GemmArgs rope_*
  EPI_ROPE = 8,
  // GeGLU backward fused into the dX GEMM of the down projection (normal orientation): v = dact[t][f] and
  // (g, u) = res[t][2f], res[t][2f+1] (the saved pre-activations): out[t][2f], [2f+1] = geglu_bwd_pair(g, u, R(v))
  EPI_GEGLU_BWD = 9,
};

// GeGLU backward of one (gate, up) pair: act = R(gelu(g)) * u, so dg = da * u * gelu'(g) and du = da * R(gelu(g))
// (gelu with the tanh approximation), packed as bf16 (dg, du).  Shared by geglu_bwd_kernel and the fused epilogue.
__device__ __forceinline__ uint32_t geglu_bwd_pair(float g, float u, float da) {
  const float s = half_one_plus_tanh(0.7978845608028654f * (g + 0.044715f * g * g * g));
  return pack_bf2(da * u * gelu_tanh_grad_s(g, s), da * rbf(g * s));
}
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
  // EPI_STORE_T
  bf16* out_t;
  int ld_out_t;
  // EPI_LORA_GRAD: D[m][c] (m = feature row, c = adapter column, adapter a = c / 16) is added to
  //   lg_trans == 0 (dB, [rows][16]):  out_f32[lg_off[a] + r_a(m) * 16 + c % 16], kept when m belongs to a
  //   lg_trans == 1 (dA, [16][lg_K]):  out_f32[lg_off[a] + (c % 16) * lg_K + m]
  // lg_mode selects which rows belong to which adapter: 0 all rows to adapter 0; 1 the q|k|v row ranges
  // (2048 | 256 | 256); 2 interleaved gate/up rows (a = m % 2, r_a = m / 2).
  int lg_mode, lg_trans, lg_K;
  long lg_off[3];
  // EPI_ROPE: token t sits at position rope_pos_off + t % rope_per_sample (rope_base[t / rope_per_sample]
  //   + t % rope_per_sample when rope_base is set).  Head blocks 0..7 (q):
  //   out[t][hb*256 + j], [.. + 128] = R(R(rope) / 16); block 8 (k): rope_k[t][j], [j+128] = R(rope);
  //   block 9 (v): rope_v[t][j], [j+128] = R(v).  rope(x1, x2) = (x1 cos - x2 sin, x2 cos + x1 sin),
  //   x1 = R(acc of dim j), x2 = R(acc of dim j+128), cos/sin tables [pos][128].
  const float* rope_cos;
  const float* rope_sin;
  int rope_pos_off, rope_per_sample, rope_ld_kv;
  const int* rope_base;  // optional: sample s's first position is rope_base[s] instead of rope_pos_off
  bf16* rope_k;
  bf16* rope_v;
  // Fused adaRMSNorm of the few-token operand (swap cluster kernel, 64-token tiles): the B tiles hold the
  // residual stream x and are normalised in shared memory before the MMAs read them,
  //   h[t][k] = R(x[t][k] * inv[t] * R(1 + nrm_scale[k]) + nrm_shift[k]),  inv[t] = 1 / sqrt(ss[t] / nrm_D + 1e-6),
  //   ss[t] = sum over p < nrm_parts of nrm_ss[p * nrm_ss_ld + t] (in order),
  // the same arithmetic as rmsnorm_kernel with its sum of squares taken from the producer's partials.
  const float* nrm_ss;
  int nrm_ss_ld, nrm_parts, nrm_D;
  const bf16* nrm_scale;
  const bf16* nrm_shift;
  // EPI_GATED in the swap cluster kernel: per-token partial sums of squares of the stored outputs, one
  // partial per 16 output features, ss_out[(f / 16) * ss_ld + t] = sum of R(out[t][f])^2.
  float* ss_out;
  int ss_ld;
};

// Extra shared memory of gemm_swap_cluster_kernel for the fused adaRMSNorm: inv[64], half sums[128],
// scale and shift of the CTA's K slice (bf16, up to 1024 features each).
constexpr int SWAP_NRM_BYTES = 256 + 512 + 2 * 1024 * 2;
constexpr int SWAP_NRM_KMAX = 1024;

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 128 ? 6 : (BN >= 64 ? 4 : 6));
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int CH = (BN % 32 == 0) ? 32 : 16;  // epilogue chunk (TMEM columns per tcgen05.ld)
};

// ---- normal orientation: one token row t, 32 consecutive features f0..f0+31 ----
template <int EPI>
__device__ __forceinline__ void epi_row32(const GemmArgs& a, float (&v)[32], int t, int f0) {
  if (t >= a.M || f0 >= a.N) return;
  const bool full = f0 + 32 <= a.N;
  if (full) {
    if (a.out_scale != 1.0f) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= a.out_scale;
    }
    if (a.bias) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float b[8];
        unpack8(reinterpret_cast<const uint4*>(a.bias + f0)[q], b);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * q + i] += b[i];
      }
    }
    if (a.addend) {
      const bf16* ad = a.addend + (size_t)(t % a.add_mod) * a.add_ld + f0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float b[8];
        unpack8(reinterpret_cast<const uint4*>(ad)[q], b);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * q + i] += b[i];
      }
    }
    if (EPI == EPI_F32) {
      float4* dst = reinterpret_cast<float4*>(a.out_f32 + (size_t)t * a.ld_out_f32 + f0);
#pragma unroll
      for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      return;
    }
    if (EPI == EPI_ROPE) {
      // columns (2j, 2j+1) of a 256-wide head block = head dims (j, j+128): 16 pairs, dims j0..j0+15
      const int hb = f0 >> 8, j0 = (f0 & 255) >> 1;
      uint32_t lo[8], hi[8];
      if (hb == 9) {
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          lo[p] = pack_bf2(v[4 * p], v[4 * p + 2]);
          hi[p] = pack_bf2(v[4 * p + 1], v[4 * p + 3]);
        }
      } else {
        const int p0 = a.rope_base ? a.rope_base[t / a.rope_per_sample] : a.rope_pos_off;
        const size_t ci = (size_t)(p0 + t % a.rope_per_sample) * 128 + j0;
        float cs[16], sn[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 c4 = reinterpret_cast<const float4*>(a.rope_cos + ci)[q];
          const float4 s4 = reinterpret_cast<const float4*>(a.rope_sin + ci)[q];
          cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
          sn[4 * q] = s4.x, sn[4 * q + 1] = s4.y, sn[4 * q + 2] = s4.z, sn[4 * q + 3] = s4.w;
        }
        const float sc = hb == 8 ? 1.0f : 0.0625f;
        float ra[16], rc[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float x1 = rbf(v[2 * p]), x2 = rbf(v[2 * p + 1]);
          ra[p] = rbf(x1 * cs[p] - x2 * sn[p]) * sc;
          rc[p] = rbf(x2 * cs[p] + x1 * sn[p]) * sc;
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          lo[p] = pack_bf2(ra[2 * p], ra[2 * p + 1]);
          hi[p] = pack_bf2(rc[2 * p], rc[2 * p + 1]);
        }
      }
      bf16* base = hb == 9 ? a.rope_v + (size_t)t * a.rope_ld_kv
                           : (hb == 8 ? a.rope_k + (size_t)t * a.rope_ld_kv : a.out + (size_t)t * a.ld_out + hb * 256);
      uint4* d0 = reinterpret_cast<uint4*>(base + j0);
      uint4* d1 = reinterpret_cast<uint4*>(base + 128 + j0);
      d0[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      d0[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
      d1[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      d1[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
      return;
    }
    if (EPI == EPI_GEGLU) {
      if (a.out_t) {
        // keep the pre-activations R(gate), R(up) (interleaved) for the backward pass
        uint4* pre = reinterpret_cast<uint4*>(a.out_t + (size_t)t * a.ld_out_t + f0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          pre[q] = make_uint4(pack_bf2(v[8 * q], v[8 * q + 1]), pack_bf2(v[8 * q + 2], v[8 * q + 3]),
                              pack_bf2(v[8 * q + 4], v[8 * q + 5]), pack_bf2(v[8 * q + 6], v[8 * q + 7]));
      }
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g0 = rbf(v[4 * j]), u0 = rbf(v[4 * j + 1]);
        const float g1 = rbf(v[4 * j + 2]), u1 = rbf(v[4 * j + 3]);
        o[j] = pack_bf2(rbf(gelu_tanh(g0)) * u0, rbf(gelu_tanh(g1)) * u1);
      }
      uint4* dst = reinterpret_cast<uint4*>(a.out + (size_t)t * a.ld_out + f0 / 2);
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
      return;
    }
    if (EPI == EPI_GEGLU_BWD) {
      const uint4* g4 = reinterpret_cast<const uint4*>(a.res + (size_t)t * a.ld_res + 2 * f0);
      uint4* dst = reinterpret_cast<uint4*>(a.out + (size_t)t * a.ld_out + 2 * f0);
      // all eight loads before the first store: the compiler cannot tell res and out apart, so a store
      // in between would hold each later load back by a full memory round trip
      uint4 gl[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) gl[q] = g4[q];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint4 gq = gl[q];
        const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 p = unpack_bf2(gw[k]);
          o[k] = geglu_bwd_pair(p.x, p.y, rbf(v[4 * q + k]));
        }
        dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      return;
    }
    if (EPI == EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(rbf(v[i]));
    }
    if (EPI == EPI_RESID || EPI == EPI_GATED) {
      const bf16* rr = a.res + (size_t)t * a.ld_res + f0;
      const bf16* gg = EPI == EPI_GATED ? a.gate + (size_t)(t / a.gate_div) * a.ld_gate + f0 : nullptr;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float r8[8];
        unpack8(reinterpret_cast<const uint4*>(rr)[q], r8);
        if (EPI == EPI_GATED) {
          float g8[8];
          unpack8(reinterpret_cast<const uint4*>(gg)[q], g8);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[8 * q + i] = r8[i] + rbf(rbf(v[8 * q + i]) * g8[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[8 * q + i] = r8[i] + rbf(v[8 * q + i]);
        }
      }
    }
    uint32_t o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = pack_bf2(v[2 * j], v[2 * j + 1]);
    uint4* dst = reinterpret_cast<uint4*>(a.out + (size_t)t * a.ld_out + f0);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
    return;
  }
  // ragged edge: scalar
#pragma unroll 1
  for (int i = 0; i < 32; ++i) {
    const int f = f0 + i;
    if (f >= a.N) break;
    float x = v[0];
#pragma unroll
    for (int k = 1; k < 32; ++k) x = (k == i) ? v[k] : x;
    x *= a.out_scale;
    if (a.bias) x += bf(a.bias[f]);
    if (a.addend) x += bf(a.addend[(size_t)(t % a.add_mod) * a.add_ld + f]);
    if (EPI == EPI_F32) {
      a.out_f32[(size_t)t * a.ld_out_f32 + f] = x;
      continue;
    }
    if (EPI == EPI_GEGLU || EPI == EPI_GEGLU_BWD) break;  // widths are multiples of 32 (checked by the host)
    if (EPI == EPI_GELU) x = gelu_tanh(rbf(x));
    if (EPI == EPI_RESID) x = bf(a.res[(size_t)t * a.ld_res + f]) + rbf(x);
    if (EPI == EPI_GATED)
      x = bf(a.res[(size_t)t * a.ld_res + f]) + rbf(rbf(x) * bf(a.gate[(size_t)(t / a.gate_div) * a.ld_gate + f]));
    a.out[(size_t)t * a.ld_out + f] = tobf(x);
  }
}

// ---- swap orientation: one feature row f, 32 consecutive tokens t0..t0+31 ----
template <int EPI>
__device__ __forceinline__ void epi_col32(const GemmArgs& a, float (&v)[32], int f, int t0) {
  const bool fok = f < a.M;
  const float bias = (fok && a.bias) ? bf(a.bias[f]) : 0.f;
  if (EPI == EPI_GEGLU) {
    // rows (2j, 2j+1) = (gate_j, up_j): the partner value lives in the neighbouring lane
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int t = t0 + i;
      const float mine = rbf(v[i] * a.out_scale + bias);
      const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
      if (fok && (f & 1) == 0 && t < a.N) a.out[(size_t)t * a.ld_out + f / 2] = tobf(rbf(gelu_tanh(mine)) * other);
    }
    return;
  }
  if (!fok) return;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int t = t0 + i;
    if (t < a.N) {
      float x = v[i] * a.out_scale + bias;
      if (EPI == EPI_F32) {
        a.out_f32[(size_t)t * a.ld_out_f32 + f] = x;
      } else {
        if (EPI == EPI_GELU) x = gelu_tanh(rbf(x));
        if (EPI == EPI_RESID) x = bf(a.res[(size_t)t * a.ld_res + f]) + rbf(x);
        if (EPI == EPI_GATED)
          x = bf(a.res[(size_t)t * a.ld_res + f]) +
              rbf(rbf(x) * bf(a.gate[(size_t)(t / a.gate_div) * a.ld_gate + f]));
        a.out[(size_t)t * a.ld_out + f] = tobf(x);
      }
    }
  }
}

// small-N epilogues (BN <= 48, normal orientation): one row, CH consecutive columns, scalar
template <int EPI, int CH>
__device__ __forceinline__ void epi_small(const GemmArgs& a, const float (&v)[32], int row, int col0) {
  if (row >= a.M) return;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = col0 + i;
    if (c >= a.N) break;
    if (EPI == EPI_LORA_GRAD) {
      const int ad = c >> 4;
      if (a.lg_trans) {
        a.out_f32[a.lg_off[ad] + (long)(c & 15) * a.lg_K + row] += v[i];
      } else {
        int owner = 0, r = row;
        if (a.lg_mode == 1) {
          owner = row < 2048 ? 0 : (row < 2304 ? 1 : 2);
          r = row - (owner == 0 ? 0 : (owner == 1 ? 2048 : 2304));
        } else if (a.lg_mode == 2) {
          owner = row & 1;
          r = row >> 1;
        }
        if (owner == ad) a.out_f32[a.lg_off[ad] + (long)r * 16 + (c & 15)] += v[i];
      }
    } else if (EPI == EPI_F32) {
      a.out_f32[(size_t)row * a.ld_out_f32 + c] = v[i] * a.out_scale;
    } else {
      const bf16 x = tobf(v[i] * a.out_scale);
      a.out[(size_t)row * a.ld_out + c] = x;
      if (EPI == EPI_STORE_T) a.out_t[(size_t)c * a.ld_out_t + row] = x;
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epi_chunk(const GemmArgs& a, float (&v)[32], int row, int col0) {
  if (a.swap)
    epi_col32<EPI>(a, v, row, col0);
  else
    epi_row32<EPI>(a, v, row, col0);
}

template <int BN, int EPI, bool AMN = false>
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
  uint64_t* tfull_bar = empty_bar + C::STAGES;  // [2] accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;          // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last split, [2] skip

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt_total = (args.K + C::BK - 1) / C::BK;
  const int n_units = args.tiles_m * args.tiles_n * args.splits;

  // a device-side wait already gave up in an earlier kernel: skip the work (uniformly for the CTA)
  if (threadIdx.x == 0) flags[2] = args.status ? *((volatile int*)args.status) : 0;
  __syncthreads();
  if (flags[2] != 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4);  // one arrival per epilogue warp
    }
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

  // unit -> (tm, tn, split, k range); splits of one tile are consecutive units
  auto decode = [&](int u, int& tm, int& tn, int& split, int& kt0, int& nkt) {
    const int tile = u / args.splits;
    split = u % args.splits;
    const int per_group = args.group_m * args.tiles_n;
    const int group = tile / per_group;
    const int first_m = group * args.group_m;
    const int gm = min(args.group_m, args.tiles_m - first_m);
    const int in_group = tile % per_group;
    tm = first_m + in_group % gm;
    tn = in_group / gm;
    kt0 = split * args.kt_per_split;
    nkt = max(0, min(kt_total, kt0 + args.kt_per_split) - kt0);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      int it = 0;
      bool waited = !args.pdl;
      for (int u = blockIdx.x; u < n_units && !flags[0]; u += gridDim.x) {
        int tm, tn, split, kt0, nkt;
        decode(u, tm, tn, split, kt0, nkt);
        for (int i = 0; i < nkt; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.status, P5_ERR_WAIT_EMPTY)) {
            flags[0] = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          if (args.swap) {
            // weights (A) never depend on the previous kernel: fetch them before waiting for it
            tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], (kt0 + i) * C::BK, tm * C::BM);
            if (!waited) {
              pdl_wait();
              waited = true;
            }
            tma_load_2d(sB + s * C::B_BYTES, &tma_b, &full_bar[s], (kt0 + i) * C::BK, tn * BN);
          } else {
            if (!waited) {
              pdl_wait();
              waited = true;
            }
            if (AMN) {
              // A is [K rows][M columns]: two boxes of 64 M-columns x 64 K-rows
              tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], tm * C::BM, (kt0 + i) * C::BK);
              tma_load_2d(sA + s * C::A_BYTES + C::A_BYTES / 2, &tma_a, &full_bar[s], tm * C::BM + 64,
                          (kt0 + i) * C::BK);
            } else {
              tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], (kt0 + i) * C::BK, tm * C::BM);
            }
            tma_load_2d(sB + s * C::B_BYTES, &tma_b, &full_bar[s], (kt0 + i) * C::BK, tn * BN);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = mma_idesc_bf16(C::BM, BN, AMN);
      int it = 0, j = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++j) {
        int tm, tn, split, kt0, nkt;
        decode(u, tm, tn, split, kt0, nkt);
        const int acc = j & 1;
        const uint32_t aph = (uint32_t)(j >> 1) & 1u;
        if (!flags[0] && !mbar_wait(&tempty_bar[acc], aph ^ 1u, args.status, P5_ERR_WAIT_ACCUM)) flags[0] = 1;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int i = 0; i < nkt && !flags[0]; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph, args.status, P5_ERR_WAIT_FULL)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES), b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {
            const uint64_t ad = AMN ? sw128_mnmajor_desc(a_addr + kk * 2048, C::A_BYTES / 2)
                                    : sw128_kmajor_desc(a_addr + kk * 32);
            tc_mma_f16(d_tmem, ad, sw128_kmajor_desc(b_addr + kk * 32), idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
        }
        tc_commit(&tfull_bar[acc]);  // accumulator complete (or abandoned on abort)
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue
    if (args.pdl) pdl_wait();
    const int sub = warp & 3;  // TMEM lanes [32*sub, 32*sub+32)
    const uint32_t lane_addr = (uint32_t)(sub * 32) << 16;
    int j = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++j) {
      int tm, tn, split, kt0, nkt;
      decode(u, tm, tn, split, kt0, nkt);
      if (EPI == EPI_GEGLU_BWD && args.splits == 1) {
        // the tile's saved pre-activations head for L2 while its MMAs run
        const int r = tm * C::BM + sub * 32 + lane, cb = tn * BN;
        if (r < args.M && cb < args.N)
          bulk_prefetch_l2(args.res + (size_t)r * args.ld_res + 2 * (size_t)cb, (uint32_t)min(BN, args.N - cb) * 4u);
      }
      const int acc = j & 1;
      const uint32_t aph = (uint32_t)(j >> 1) & 1u;
      const bool ok = mbar_wait(&tfull_bar[acc], aph, args.status, P5_ERR_WAIT_ACCUM) && !flags[0] && nkt > 0;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_addr + (uint32_t)(acc * BN);
      const int row = tm * C::BM + sub * 32 + lane;
      const int col_base = tn * BN;
      if (EPI == EPI_GEGLU_BWD && args.splits == 1) {
        // software-pipelined: chunk c + 32's saved pre-activations (8 x 16 bytes per thread) are in flight
        // while chunk c computes; rows past M read row M - 1 and store nothing
        const int cmax = min(BN, args.N - col_base);
        const uint4* gsrc =
            reinterpret_cast<const uint4*>(args.res + (size_t)min(row, args.M - 1) * args.ld_res + 2 * (size_t)col_base);
        uint4 gc[8], gn[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          gc[q] = ok ? gsrc[q] : make_uint4(0u, 0u, 0u, 0u);
          gn[q] = gc[q];
        }
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          const bool live = ok && c < cmax;
          if (live && c + 32 < cmax) {
#pragma unroll
            for (int q = 0; q < 8; ++q) gn[q] = gsrc[(c + 32) / 4 + q];
          }
          uint32_t r[32];
          tmem_ld32(t_acc + (uint32_t)c, r);
          tmem_wait_ld();
          if (live && row < args.M) {
            uint4* dst = reinterpret_cast<uint4*>(args.out + (size_t)row * args.ld_out + 2 * (size_t)(col_base + c));
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const uint32_t gw[4] = {gc[q].x, gc[q].y, gc[q].z, gc[q].w};
              uint32_t o[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 p = unpack_bf2(gw[k]);
                o[k] = geglu_bwd_pair(p.x, p.y, rbf(__uint_as_float(r[4 * q + k])));
              }
              dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) gc[q] = gn[q];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      } else if (args.splits == 1) {
#pragma unroll 1
        for (int c = 0; c < BN; c += C::CH) {
          uint32_t r[32];
          if (C::CH == 32) {
            tmem_ld32(t_acc + (uint32_t)c, r);
          } else {
            tmem_ld16(t_acc + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = (ok && i < C::CH) ? __uint_as_float(r[i]) : 0.f;
          if (ok) {
            if (BN < 64)
              epi_small<EPI, C::CH>(args, v, row, col_base + c);
            else
              epi_chunk<EPI>(args, v, row, col_base + c);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      } else {
        // split-K: partial tile to the workspace, ticket, the last split reduces in split order
        const int tile_id = tm * args.tiles_n + tn;
        const size_t tile_elems = (size_t)C::BM * BN;
        const int lrow = sub * 32 + lane;
        float* mine = args.ws + ((size_t)split * args.tiles_m * args.tiles_n + tile_id) * tile_elems + (size_t)lrow * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += C::CH) {
          uint32_t r[32];
          if (C::CH == 32) {
            tmem_ld32(t_acc + (uint32_t)c, r);
          } else {
            tmem_ld16(t_acc + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(mine + c);
#pragma unroll
          for (int q = 0; q < C::CH / 4; ++q)
            dst[q] = ok ? make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                      __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);  // accumulator free for the next unit
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 128) {
          const int prev = atomicAdd(&args.counters[tile_id], 1);
          flags[1] = (prev == args.splits - 1) ? 1 : 0;
          if (prev == args.splits - 1) args.counters[tile_id] = 0;  // re-arm for the next launch
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (flags[1]) {
          __threadfence();
          const float* base = args.ws + (size_t)tile_id * tile_elems + (size_t)lrow * BN;
          const size_t sstride = (size_t)args.tiles_m * args.tiles_n * tile_elems;
#pragma unroll 1
          for (int c = 0; c < BN; c += C::CH) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
            // four splits' loads in flight per round; the sums still run in split order
            int s = 0;
#pragma unroll 1
            for (; s + 4 <= args.splits; s += 4) {
              float4 p[4][8];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float4* src = reinterpret_cast<const float4*>(base + (s + h) * sstride + c);
#pragma unroll
                for (int q = 0; q < C::CH / 4; ++q) p[h][q] = __ldcg(src + q);
              }
#pragma unroll
              for (int h = 0; h < 4; ++h)
#pragma unroll
                for (int q = 0; q < C::CH / 4; ++q) {
                  v[4 * q] += p[h][q].x;
                  v[4 * q + 1] += p[h][q].y;
                  v[4 * q + 2] += p[h][q].z;
                  v[4 * q + 3] += p[h][q].w;
                }
            }
#pragma unroll 1
            for (; s < args.splits; ++s) {
              const float4* src = reinterpret_cast<const float4*>(base + s * sstride + c);
#pragma unroll
              for (int q = 0; q < C::CH / 4; ++q) {
                const float4 p = __ldcg(src + q);
                v[4 * q] += p.x;
                v[4 * q + 1] += p.y;
                v[4 * q + 2] += p.z;
                v[4 * q + 3] += p.w;
              }
            }
            if (BN < 64)
              epi_small<EPI, C::CH>(args, v, row, col_base + c);
            else
              epi_chunk<EPI>(args, v, row, col_base + c);
          }
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

// ---------------------------------------------------------------------------------------------------
// Few-token weight streaming with split-K inside a thread-block cluster (swap orientation only).
//
// A tile of 128 weight rows x BN tokens (BN <= 256; several token tiles for up to ~1000 tokens) is
// split along K over the S CTAs of one cluster (S <= 8).  Each CTA
// stages its fp32 partial tile in its own shared memory; after a cluster barrier CTA r reduces rows
// [r*128/S, (r+1)*128/S) by reading the S partials over distributed shared memory in rank order
// (deterministic), applies the epilogue and stores.  The partials never leave the chip and the
// reduction is spread over all S CTAs instead of the last one.

// Epilogue operands of one reduce item (weight row f, tokens t0..t0+3), loaded from global memory
// before the partial sums are: they do not depend on them.
struct SwapEpiOps {
  float bias, res[4], gate[4];
};
// Epilogue operands of item (row f, tokens t0..t0+3).  Rows and tokens past the extents read the last
// valid row / token instead (never stored): the loads carry no conditions, so all of them are in
// flight together (measured: eight guarded loads took ~2,800 cycles, one L2 round trip is ~500).
template <int EPI>
__device__ __forceinline__ void swap_epi_load(const GemmArgs& a, int f, int t0, SwapEpiOps& o) {
  const int fc = min(f, a.M - 1);
  o.bias = a.bias ? bf(a.bias[fc]) : 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int tc = min(t0 + q, a.N - 1);
    if (EPI == EPI_ROPE) {  // res, gate carry cos, sin of the token's position for this row pair
      const int p0 = a.rope_base ? a.rope_base[tc / a.rope_per_sample] : a.rope_pos_off;
      const size_t ci = (size_t)(p0 + tc % a.rope_per_sample) * 128 + ((fc & 255) >> 1);
      o.res[q] = a.rope_cos[ci];
      o.gate[q] = a.rope_sin[ci];
    } else {
      o.res[q] = (EPI == EPI_RESID || EPI == EPI_GATED) ? bf(a.res[(size_t)tc * a.ld_res + fc]) : 0.f;
      o.gate[q] = EPI == EPI_GATED ? bf(a.gate[(size_t)(tc / a.gate_div) * a.ld_gate + fc]) : 0.f;
    }
  }
}
template <int EPI>
__device__ __forceinline__ float swap_epi_value(const GemmArgs& a, float v, const SwapEpiOps& o, int q) {
  const float x = v * a.out_scale + o.bias;
  if (EPI == EPI_F32) return x;
  if (EPI == EPI_GELU) return gelu_tanh(rbf(x));
  if (EPI == EPI_RESID) return o.res[q] + rbf(x);
  if (EPI == EPI_GATED) return o.res[q] + rbf(rbf(x) * o.gate[q]);
  return x;
}

// Cluster reduce of a swap-orientation tile: CTA `rank` of S owns rows [rank*R, rank*R+R), R = 128/S.
// Items = (row, group of 4 tokens); consecutive threads take consecutive weight rows of one group, so
// the stores of each token are contiguous across the warp (R*BN/4 is a multiple of 256: all eight
// warps of the CTA take part).  The partials are summed in rank order (deterministic).
//   PUSH: every CTA has already sent row slice p of its partial tile to CTA p with one bulk copy
//     (recv slot = source rank); an item's epilogue operands (bias, residual, gate) are requested from
//     global memory, then the thread waits for the S-1 incoming slices (first item only), arrives on the
//     cluster barrier that guards the copies' source buffers, and sums from its own shared memory.
//     Measured on B200: S scattered 16-byte loads per thread from the peers' shared memory are bound
//     by the request rate (~6,000 cycles for S = 8); S-1 bulk copies of R rows each are not.
//   otherwise (tiles too wide for a second partial buffer): S direct loads from the peers' memory.
template <int BN, int EPI, int S, bool PUSH>
__device__ __forceinline__ void swap_reduce(const GemmArgs& args, uint32_t red_base, const float* red,
                                            const float* recv, uint64_t* recv_bar, int rank, int m0, int n0,
                                            int rtid) {
  constexpr int R = 128 / S, RED_LD = BN + 4, ITEMS = R * (BN / 4);
  static_assert(ITEMS >= 256, "every thread must take a first item (it arrives on the cluster barrier there)");
  // GeGLU (gate, up) and RoPE (dim j, dim j+128) rows come in neighbouring pairs: one item per pair and
  // 4 tokens when that still gives every thread a first item (no shuffles, every lane stores)
  constexpr int RP = R / 2, ITEMS_P = RP * (BN / 4);
  constexpr bool PAIR = (EPI == EPI_GEGLU || EPI == EPI_ROPE) && ITEMS_P >= 256;
  if (PAIR) {
#pragma unroll 1
    for (int it = rtid; it < ITEMS_P; it += 256) {
      const int lp = it % RP, cg = it / RP;
      const int lr = 2 * lp, f = m0 + rank * R + lr;  // even row of the pair
      SwapEpiOps o;
      swap_epi_load<EPI>(args, f, n0 + cg * 4, o);
      const float bias1 = (EPI == EPI_GEGLU && args.bias) ? bf(args.bias[min(f + 1, args.M - 1)]) : 0.f;
      float4 pa[S], pb[S];
      if (PUSH) {
        if (it == rtid) {
          mbar_wait(recv_bar, 0, args.status, P5_ERR_WAIT_FULL);
          cluster_arrive_relaxed();  // the copies into this CTA have landed
        }
#pragma unroll
        for (int p = 0; p < S; ++p) {
          const float* src = p == rank ? red + (rank * R + lr) * RED_LD : recv + (p * R + lr) * RED_LD;
          pa[p] = *reinterpret_cast<const float4*>(src + cg * 4);
          pb[p] = *reinterpret_cast<const float4*>(src + RED_LD + cg * 4);
        }
      } else {
        const uint32_t addr = red_base + (uint32_t)((rank * R + lr) * RED_LD + cg * 4) * 4u;
#pragma unroll
        for (int p = 0; p < S; ++p) {
          pa[p] = ld_peer_v4(map_peer(addr, (uint32_t)p));
          pb[p] = ld_peer_v4(map_peer(addr + RED_LD * 4u, (uint32_t)p));
        }
      }
      float va[4] = {0.f, 0.f, 0.f, 0.f}, vb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < S; ++p) {
        va[0] += pa[p].x;
        va[1] += pa[p].y;
        va[2] += pa[p].z;
        va[3] += pa[p].w;
        vb[0] += pb[p].x;
        vb[1] += pb[p].y;
        vb[2] += pb[p].z;
        vb[3] += pb[p].w;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = n0 + cg * 4 + q;
        if (f >= args.M || t >= args.N) continue;
        if (EPI == EPI_GEGLU) {
          const float gt = rbf(va[q] * args.out_scale + o.bias), up = rbf(vb[q] * args.out_scale + bias1);
          args.out[(size_t)t * args.ld_out + f / 2] = tobf(rbf(gelu_tanh(gt)) * up);
        } else {
          const float x1 = rbf(va[q]), x2 = rbf(vb[q]);
          const int hb = f >> 8, j = (f & 255) >> 1;
          if (hb == 9) {
            args.rope_v[(size_t)t * args.rope_ld_kv + j] = tobf(x1);
            args.rope_v[(size_t)t * args.rope_ld_kv + j + 128] = tobf(x2);
          } else {
            const float cs = o.res[q], sn = o.gate[q];
            const float ra = rbf(x1 * cs - x2 * sn);
            const float rc = rbf(x2 * cs + x1 * sn);
            if (hb == 8) {
              args.rope_k[(size_t)t * args.rope_ld_kv + j] = tobf(ra);
              args.rope_k[(size_t)t * args.rope_ld_kv + j + 128] = tobf(rc);
            } else {
              args.out[(size_t)t * args.ld_out + hb * 256 + j] = tobf(ra * 0.0625f);
              args.out[(size_t)t * args.ld_out + hb * 256 + j + 128] = tobf(rc * 0.0625f);
            }
          }
        }
      }
    }
    return;
  }
#pragma unroll 1
  for (int it = rtid; it < ITEMS; it += 256) {
    const int lr = it % R, cg = it / R;
    const int f = m0 + rank * R + lr;
    SwapEpiOps o;
    swap_epi_load<EPI>(args, f, n0 + cg * 4, o);
    float4 pv[S];
    if (PUSH) {
      if (it == rtid) {
        mbar_wait(recv_bar, 0, args.status, P5_ERR_WAIT_FULL);
        cluster_arrive_relaxed();  // the copies into this CTA have landed
      }
#pragma unroll
      for (int p = 0; p < S; ++p)
        pv[p] = p == rank ? *reinterpret_cast<const float4*>(red + (rank * R + lr) * RED_LD + cg * 4)
                          : *reinterpret_cast<const float4*>(recv + (p * R + lr) * RED_LD + cg * 4);
    } else {
      const uint32_t addr = red_base + (uint32_t)((rank * R + lr) * RED_LD + cg * 4) * 4u;
#pragma unroll
      for (int p = 0; p < S; ++p) pv[p] = ld_peer_v4(map_peer(addr, (uint32_t)p));
    }
    float v[4] = {0.f, 0.f, 0.f, 0.f}, sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < S; ++p) {
      v[0] += pv[p].x;
      v[1] += pv[p].y;
      v[2] += pv[p].z;
      v[3] += pv[p].w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int t = n0 + cg * 4 + q;
      const bool valid = f < args.M && t < args.N;
      if (EPI == EPI_GEGLU) {
        // rows (2j, 2j+1) = (gate_j, up_j) sit in neighbouring lanes (R is even)
        const float mine = rbf(v[q] * args.out_scale + o.bias);
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        if (valid && (f & 1) == 0) args.out[(size_t)t * args.ld_out + f / 2] = tobf(rbf(gelu_tanh(mine)) * other);
      } else if (EPI == EPI_ROPE) {
        // rows (2j, 2j+1) of a head block = dims (j, j+128), in neighbouring lanes
        const float mine = rbf(v[q]);
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        if (valid && (f & 1) == 0) {
          const int hb = f >> 8, j = (f & 255) >> 1;
          if (hb == 9) {
            args.rope_v[(size_t)t * args.rope_ld_kv + j] = tobf(mine);
            args.rope_v[(size_t)t * args.rope_ld_kv + j + 128] = tobf(other);
          } else {
            const float cs = o.res[q], sn = o.gate[q];
            const float ra = rbf(mine * cs - other * sn);
            const float rc = rbf(other * cs + mine * sn);
            if (hb == 8) {
              args.rope_k[(size_t)t * args.rope_ld_kv + j] = tobf(ra);
              args.rope_k[(size_t)t * args.rope_ld_kv + j + 128] = tobf(rc);
            } else {
              args.out[(size_t)t * args.ld_out + hb * 256 + j] = tobf(ra * 0.0625f);
              args.out[(size_t)t * args.ld_out + hb * 256 + j + 128] = tobf(rc * 0.0625f);
            }
          }
        }
      } else if (valid) {
        const float x = swap_epi_value<EPI>(args, v[q], o, q);
        if (EPI == EPI_F32) {
          args.out_f32[(size_t)t * args.ld_out_f32 + f] = x;
        } else {
          const bf16 xb = tobf(x);
          args.out[(size_t)t * args.ld_out + f] = xb;
          sq[q] = bf(xb) * bf(xb);
        }
      }
    }
    if (EPI == EPI_GATED && args.ss_out) {
      // 16 consecutive lanes hold 16 consecutive features f of the same 4 tokens (R >= 16)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int o2 = 8; o2; o2 >>= 1) sq[q] += __shfl_xor_sync(0xffffffffu, sq[q], o2);
      }
      if ((rtid & 15) == 0 && f < args.M) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int t = n0 + cg * 4 + q;
          if (t < args.N) args.ss_out[(size_t)(f >> 4) * args.ss_ld + t] = sq[q];
        }
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(256, 2)
    gemm_swap_cluster_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                             const GemmArgs args) {
  using C = GemmCfg<BN>;
  constexpr int RED_LD = BN + 4;  // fp32 partial row stride: 16-byte rows, 8 rows hit 8 distinct 16-byte slots
  static_assert(128 * RED_LD * 4 <= C::STAGES * C::STAGE_BYTES, "partial tile must fit in the stage buffers");
  // second tile-sized buffer (received slices) behind the partial tile, also in the stage buffers
  constexpr bool PUSH = 2 * 128 * RED_LD * 4 <= C::STAGES * C::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  float* red = reinterpret_cast<float*>(smem);  // reuses the stage buffers once the MMAs are done
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* accum_bar = empty_bar + C::STAGES;
  uint64_t* ready_bar = accum_bar + 1;  // fused adaRMSNorm: B stage normalised in place
  uint64_t* recv_bar = ready_bar + C::STAGES;  // partial-tile slices from the other CTAs of the cluster
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* nrm_inv = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);  // [64]
  float* nrm_half = nrm_inv + 64;                                                      // [2][64]
  bf16* nrm_sc = reinterpret_cast<bf16*>(nrm_half + 128);                              // [SWAP_NRM_KMAX]
  bf16* nrm_sh = nrm_sc + SWAP_NRM_KMAX;
  const bool nrm = BN == 64 && args.nrm_ss != nullptr;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = (int)cluster_size(), rank = (int)cluster_rank();
  const int tile = blockIdx.x / S;  // clusters walk the weight tiles first, then the token tiles
  const int tm = tile % args.tiles_m, tn = tile / args.tiles_m;
  const int m0 = tm * C::BM, n0 = tn * BN;
  const int kt_total = (args.K + C::BK - 1) / C::BK;
  const int kt0 = rank * args.kt_per_split;
  const int nkt = max(0, min(kt_total, kt0 + args.kt_per_split) - kt0);
  constexpr uint32_t TCOLS = BN < 32 ? 32 : BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accum_bar, 1);
    if (nrm)
      for (int s = 0; s < C::STAGES; ++s) mbar_init(&ready_bar[s], 128);
    mbar_init(recv_bar, 1);
    flags[0] = 0;
    fence_barrier_init();
    if (PUSH) mbar_arrive_expect_tx(recv_bar, (uint32_t)(S - 1) * (128 / S) * RED_LD * 4);
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (args.pdl) pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      bool waited = !args.pdl;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.status, P5_ERR_WAIT_EMPTY)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
        tma_load_2d(sA + s * C::A_BYTES, &tma_a, &full_bar[s], (kt0 + i) * C::BK, m0);  // weights: no dependency
        if (!waited) {
          pdl_wait();
          waited = true;
        }
        tma_load_2d(sB + s * C::B_BYTES, &tma_b, &full_bar[s], (kt0 + i) * C::BK, n0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = mma_idesc_bf16(C::BM, BN);
      for (int i = 0; i < nkt && !flags[0]; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait(nrm ? &ready_bar[s] : &full_bar[s], ph, args.status, P5_ERR_WAIT_FULL)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES), b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32), idesc,
                     (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty_bar[s]);
      }
      tc_commit(accum_bar);
    }
    __syncwarp();
  } else if (warp >= 4) {
    if (nrm) {
      // ---- fused adaRMSNorm: per-token inverse RMS from the producer's partials, then each B stage
      // (64 token rows x 64 features, 128-byte swizzled rows) is normalised in place before the MMAs
      const int nt = threadIdx.x - 128, tt = nt & 63, half = nt >> 6;
      if (args.pdl) pdl_wait();
      // every global load is issued before the first shared-memory store (the compiler cannot tell
      // them apart, so a store in between would hold the later loads back by a round trip); tokens
      // past the tile's extent read the last token's partials (never used), so the loads carry no
      // conditions.  The K slice has at most SWAP_NRM_KMAX features: one 8-feature chunk per thread.
      const int kbase = kt0 * C::BK, nch = nkt * C::BK / 8;
      const int hp = args.nrm_parts / 2, p0 = half * hp;
      const float* src = args.nrm_ss + (size_t)p0 * args.nrm_ss_ld + min(n0 + tt, args.N - 1);
      float acc = 0.f;
      const int kb = nch > 0 ? kbase : 0, cc = nch > 0 ? min(nt, nch - 1) : 0;  // a split without K tiles reads chunk 0
      const uint4 scv = reinterpret_cast<const uint4*>(args.nrm_scale + kb)[cc];
      const uint4 shv = reinterpret_cast<const uint4*>(args.nrm_shift + kb)[cc];
      if (hp == 32) {
        float v[32];
#pragma unroll
        for (int p = 0; p < 32; ++p) v[p] = src[(size_t)p * args.nrm_ss_ld];
#pragma unroll
        for (int p = 0; p < 32; ++p) acc += v[p];
      } else {
#pragma unroll 8
        for (int p = 0; p < hp; ++p) acc += src[(size_t)p * args.nrm_ss_ld];
      }
      if (nt < nch) {
        reinterpret_cast<uint4*>(nrm_sc)[nt] = scv;
        reinterpret_cast<uint4*>(nrm_sh)[nt] = shv;
      }
      nrm_half[nt] = acc;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (nt < 64)
        nrm_inv[nt] = n0 + nt < args.N ? 1.0f / sqrtf((nrm_half[nt] + nrm_half[64 + nt]) / (float)args.nrm_D + 1e-6f)
                                       : 0.f;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // thread nt owns 16-byte chunk position pc of rows r0 + 16j; with the 128-byte swizzle those hold
      // the same 8 features lc of every K block
      const int pc = nt & 7, r0 = nt >> 3, lc = pc ^ (r0 & 7);
      for (int i = 0; i < nkt && !flags[0]; ++i) {
        const int s = i % C::STAGES;
        if (!mbar_wait(&full_bar[s], (uint32_t)(i / C::STAGES) & 1u, args.status, P5_ERR_WAIT_FULL)) {
          flags[0] = 1;
          break;
        }
        float sc[8], sh[8];
        unpack8(reinterpret_cast<const uint4*>(nrm_sc)[i * 8 + lc], sc);
        unpack8(reinterpret_cast<const uint4*>(nrm_sh)[i * 8 + lc], sh);
#pragma unroll
        for (int q = 0; q < 8; ++q) sc[q] = rbf(1.0f + sc[q]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = r0 + 16 * j;
          uint4* ptr = reinterpret_cast<uint4*>(sB + s * C::B_BYTES + r * 128 + pc * 16);
          float xv[8];
          unpack8(*ptr, xv);
          const float inv = nrm_inv[r];
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = xv[2 * q] * inv * sc[2 * q] + sh[2 * q];
            const float a1 = xv[2 * q + 1] * inv * sc[2 * q + 1] + sh[2 * q + 1];
            w[q] = inv != 0.f ? pack_bf2(a0, a1) : 0u;
          }
          *ptr = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
        mbar_arrive(&ready_bar[s]);
      }
    }
    // partial tile -> own shared memory (zeros when this split had no K-tiles or gave up)
    const int sub = warp & 3;
    const bool ok = mbar_wait(accum_bar, 0, args.status, P5_ERR_WAIT_ACCUM) && !flags[0] && nkt > 0;
    tc_fence_after();
    const int row = sub * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)c, r);
      tmem_wait_ld();
      float4* dst = reinterpret_cast<float4*>(red + row * RED_LD + c);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = ok ? make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                  __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (PUSH) fence_proxy_async_smem();  // the partial tile is the source of bulk copies
  }
  tc_fence_before();
  cluster_sync();  // every partial tile of the cluster is in shared memory, every CTA's MMAs are done

  const uint32_t red_base = smem_u32(red);
  const float* recv = red + 128 * RED_LD;
  if (PUSH && warp == 0 && lane < S && lane != rank) {
    // rows [lane*R, lane*R+R) of this CTA's partial -> slot `rank` of CTA `lane`'s receive buffer
    const uint32_t slice = (uint32_t)(128 / S) * RED_LD * 4;
    bulk_copy_to_peer(map_peer(smem_u32(recv) + (uint32_t)rank * slice, (uint32_t)lane),
                      red_base + (uint32_t)lane * slice, slice, map_peer(smem_u32(recv_bar), (uint32_t)lane));
  }
  {  // all eight warps reduce (the producer and MMA warps are done by now)
    if (args.pdl) pdl_wait();
    const int rtid = threadIdx.x;
    switch (S) {
      case 2: swap_reduce<BN, EPI, 2, PUSH>(args, red_base, red, recv, recv_bar, rank, m0, n0, rtid); break;
      case 4: swap_reduce<BN, EPI, 4, PUSH>(args, red_base, red, recv, recv_bar, rank, m0, n0, rtid); break;
      case 8: swap_reduce<BN, EPI, 8, PUSH>(args, red_base, red, recv, recv_bar, rank, m0, n0, rtid); break;
      default: swap_reduce<BN, EPI, 1, PUSH>(args, red_base, red, recv, recv_bar, rank, m0, n0, rtid); break;
    }
  }
  // PUSH: every CTA's incoming copies have landed, so this CTA's outgoing copies have read their source;
  // otherwise: the peers are done reading this CTA's partial tile
  if (PUSH)
    cluster_wait_acquire();
  else
    cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

}  // namespace p5

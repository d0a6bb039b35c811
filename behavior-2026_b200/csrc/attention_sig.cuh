// attention_sig.cuh — SigLIP multi-head attention (16 heads of 72 within each 256-token image) on tcgen05.
//
// Same contract as attn_kernel<72> for SigLIP (q <- R(q / qdiv), keys = the image's 256 tokens, fp32
// logits and softmax, P rounded to bf16 for P V, l the sum of the fp32 P), re-tiled for the 5th-generation
// tensor cores:
//   * a CTA owns 128 queries of one head of one image; all 256 keys fit one S tile, so the softmax is
//     exact (one max, no online rescaling);
//   * head_dim 72 is padded to 80 with zeros (the MMA K step is 16) in 128-byte-swizzled shared memory,
//     filled by plain 16-byte loads (a 144-byte head row does not fit a 128-byte TMA swizzle box);
//   * TMEM (512 columns): S = Q K^T (M=128, N=256) in columns 0-255, P (bf16, two per column) in 256-383
//     as the A operand of O = P V, O (N=80, V read MN-major from its [key][dim] rows) in 384-463;
//   * two softmax warpgroups, thread = query row = TMEM lane, each half of the keys; the two row maxima
//     meet through shared memory.
#pragma once
#include "attention.cuh"

namespace p5 {

struct AttnSigCfg {
  static constexpr int ROWS = 128, KEYS = 256, HD = 72, CH = 9;  // 16-byte chunks of a head row
  static constexpr int Q_KB = ROWS * 128;                        // one 64-dim block of Q: 16 KB
  static constexpr int K_KB = KEYS * 128;                        // one 64-dim block of K or V: 32 KB
  static constexpr int Q_OFF = 0, K_OFF = 2 * Q_KB, V_OFF = K_OFF + 2 * K_KB;
  static constexpr int BAR_OFF = V_OFF + 2 * K_KB;               // 160 KB
  static constexpr int SMEM = 1024 + BAR_OFF + 2048 + 256;
  static constexpr int S_COL = 0, P_COL = 256, O_COL = 384, TMEM_COLS = 512;
};

// byte offset of 16-byte chunk c (of 10: dims 8c..8c+7, chunk 9 = zero pad) of row `row` in a buffer of
// 64-dim blocks of `rows` rows x 128 bytes, 128-byte swizzle
__device__ __forceinline__ uint32_t sig_chunk_off(int row, int c, int block_bytes) {
  return (uint32_t)((c >> 3) * block_bytes + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(384, 1) attn_sig_kernel(const AttnArgs a, int* status) {
  using C = AttnSigCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint64_t* s_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = s_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 3);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xm = reinterpret_cast<float*>(smem + C::BAR_OFF + 64);  // [2][128] row maxima
  float* lx = xm + 2 * C::ROWS;                                   // [2][128] row sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int rb = blockIdx.x, h = blockIdx.y, img = blockIdx.z;

  if (tid == 0) flags[0] = status ? *((volatile int*)status) : 0;
  __syncthreads();
  if (flags[0] != 0) return;
  if (tid == 0) {
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);  // one arrival per softmax warp
    mbar_init(o_full, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }

  // ---- Q (scaled: R(q / qdiv)), K, V -> swizzled shared memory; dims 72..79 zero
  if (a.pdl) pdl_wait();
  const bf16* qb = a.q + img * a.q_bstride + (long)(rb * C::ROWS) * a.ldq + h * C::HD;
  const bf16* kb = a.k1 + img * a.b1stride + h * C::HD;
  const bf16* vb = a.v1 + img * a.b1stride + h * C::HD;
  for (int i = tid; i < C::KEYS * 10; i += blockDim.x) {
    const int key = i / 10, c = i % 10;
    const uint32_t ko = sig_chunk_off(key, c, C::K_KB);
    if (c < C::CH) {
      cp_async16(sK + ko, kb + (long)key * a.ld1 + c * 8, true);
      cp_async16(sV + ko, vb + (long)key * a.ld1 + c * 8, true);
    } else {
      *reinterpret_cast<uint4*>(sK + ko) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(sV + ko) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  cp_async_commit();
  for (int i = tid; i < C::ROWS * 10; i += blockDim.x) {
    const int r = i / 10, c = i % 10;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (c < C::CH) {
      const uint4 u = *reinterpret_cast<const uint4*>(qb + (long)r * a.ldq + c * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      uint32_t t[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf2(w[k]);
        t[k] = pack_bf2(f.x / a.qdiv, f.y / a.qdiv);
      }
      o = make_uint4(t[0], t[1], t[2], t[3]);
    }
    *reinterpret_cast<uint4*>(sQ + sig_chunk_off(r, c, C::Q_KB)) = o;
  }
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (a.pdl) pdl_launch_dependents();

  // ---- S = Q K^T (K = 80: four steps in dims 0-63, one in 64-79)
  if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::KEYS);
    const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
    for (int kk = 0; kk < 5; ++kk)
      tc_mma_f16(tmem_base + C::S_COL, sw128_kmajor_desc(qa + (kk >> 2) * C::Q_KB + (kk & 3) * 32),
                 sw128_kmajor_desc(ka + (kk >> 2) * C::K_KB + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
    tc_commit(s_full);
  }

  // ---- softmax: warpgroup g owns keys [128g, 128g+128) of row r
  const int g = (warp - 4) >> 2, sub = warp & 3, r = sub * 32 + lane;
  const uint32_t t_lane = tmem_base + ((uint32_t)(sub * 32) << 16);
  float l_part = 0.f;
  if (warp >= 4) {
    mbar_wait(s_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32(t_lane + (uint32_t)(C::S_COL + g * 128 + c * 32), v);
      tmem_wait_ld();
      float m4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        m4[k] = fmax3(__uint_as_float(v[8 * k]), __uint_as_float(v[8 * k + 1]),
                      fmax3(__uint_as_float(v[8 * k + 2]), __uint_as_float(v[8 * k + 3]),
                            fmax3(__uint_as_float(v[8 * k + 4]), __uint_as_float(v[8 * k + 5]),
                                  fmaxf(__uint_as_float(v[8 * k + 6]), __uint_as_float(v[8 * k + 7])))));
      mx = fmax3(mx, fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    }
    xm[g * C::ROWS + r] = mx;
    asm volatile("bar.sync %0, 64;" ::"r"(1 + sub) : "memory");  // the two warps of this row group
    const float msc = fmaxf(xm[r], xm[C::ROWS + r]) * LOG2E;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32(t_lane + (uint32_t)(C::S_COL + g * 128 + c * 32), v);
      tmem_wait_ld();
      uint32_t pk[16];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(v[2 * k]), LOG2E, -msc));
        const float p1 = ex2_approx(fmaf(__uint_as_float(v[2 * k + 1]), LOG2E, -msc));
        ls[k & 3] += p0 + p1;
        pk[k] = pack_bf2(p0, p1);
      }
      l_part += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_st16(t_lane + (uint32_t)(C::P_COL + g * 64 + c * 16), pk);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full);
  }

  // ---- O = P V (P from TMEM, V MN-major: two 64-dim blocks 32 KB apart, 16 keys per step)
  if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc_o = mma_idesc_bf16(128, 80, false, true);
    const bool ok = mbar_wait(p_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    const uint32_t va = smem_u32(sV);
    if (ok) {
#pragma unroll
      for (int kk = 0; kk < C::KEYS / 16; ++kk)
        tc_mma_f16_ta(tmem_base + C::O_COL, tmem_base + (uint32_t)(C::P_COL + kk * 8),
                      sw128_mnmajor_desc(va + kk * 2048, C::K_KB), idesc_o, kk > 0 ? 1u : 0u);
    }
    tc_commit(o_full);
  }

  // ---- epilogue: out = O / l (warpgroup 0 stores the 72 dims of its rows)
  if (warp >= 4) {
    lx[g * C::ROWS + r] = l_part;
    asm volatile("bar.sync 5, 256;" ::: "memory");
    const float l = lx[r] + lx[C::ROWS + r];
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    const bool done = mbar_wait(o_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    if (g == 0) {
      uint32_t o0[32], o1[32], o2[16];
      tmem_ld32(t_lane + C::O_COL, o0);
      tmem_ld32(t_lane + C::O_COL + 32, o1);
      tmem_ld16(t_lane + C::O_COL + 64, o2);
      tmem_wait_ld();
      if (done) {
        uint4* dst = reinterpret_cast<uint4*>(a.out + img * a.o_bstride + (long)(rb * C::ROWS + r) * a.ldo + h * C::HD);
        auto pk = [&](float x, float y) { return pack_bf2(x * inv, y * inv); };
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pk(__uint_as_float(o0[8 * q]), __uint_as_float(o0[8 * q + 1])),
                              pk(__uint_as_float(o0[8 * q + 2]), __uint_as_float(o0[8 * q + 3])),
                              pk(__uint_as_float(o0[8 * q + 4]), __uint_as_float(o0[8 * q + 5])),
                              pk(__uint_as_float(o0[8 * q + 6]), __uint_as_float(o0[8 * q + 7])));
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[4 + q] = make_uint4(pk(__uint_as_float(o1[8 * q]), __uint_as_float(o1[8 * q + 1])),
                                  pk(__uint_as_float(o1[8 * q + 2]), __uint_as_float(o1[8 * q + 3])),
                                  pk(__uint_as_float(o1[8 * q + 4]), __uint_as_float(o1[8 * q + 5])),
                                  pk(__uint_as_float(o1[8 * q + 6]), __uint_as_float(o1[8 * q + 7])));
        dst[8] = make_uint4(pk(__uint_as_float(o2[0]), __uint_as_float(o2[1])),
                            pk(__uint_as_float(o2[2]), __uint_as_float(o2[3])),
                            pk(__uint_as_float(o2[4]), __uint_as_float(o2[5])),
                            pk(__uint_as_float(o2[6]), __uint_as_float(o2[7])));
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

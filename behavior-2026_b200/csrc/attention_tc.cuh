// attention_tc.cuh — MQA attention with head_dim 256 on the 5th-generation tensor cores.
//
// Same contract as attn_kernel<256> for the Gemma prefix and the action expert (8 query heads folded
// into rows, one shared K/V head, keys = [segment 1 || segment 2], optional split-KV partials and
// log-sum-exp), re-tiled for tcgen05:
//
//   * a CTA owns 128 query rows (16 tokens x 8 heads).  Q (128 x 256 bf16, 64 KB) is loaded once by
//     a 4-D TMA box per 64-column block into 128-byte-swizzled K-major shared memory;
//   * keys are walked in tiles of 64 that never straddle the two segments (each segment is its own
//     3-D tensor map; rows past a segment end are zero-filled by TMA and masked in the softmax);
//   * one thread issues S = Q K^T (M=128, N=64, K=256) into one of two TMEM buffers and
//     O += P V (M=128, N=256, K=64) into a 256-column TMEM accumulator; V is consumed MN-major
//     straight from its [key][dim] layout, P is written to shared memory by the softmax threads;
//   * K and V tiles share one 4-slot TMA ring, loaded in the order the MMA thread consumes them
//     (K0, K1, V0, K2, V1, ...), so S for tile j+1 runs on the tensor cores while tile j's softmax runs;
//   * two softmax warpgroups (8 warps, two per SM sub-partition to hide each other's latency); a
//     thread owns one row (one TMEM lane) and half of the tile's 64 columns, and reads the other half
//     only for the row max, so the two halves agree on the running max without exchanging it.
//     The running max is only moved (and O rescaled through tcgen05.ld/st) when a tile's max exceeds
//     it by more than 2^8 in the exponent, so P stays <= 256 and O is rarely touched.
// Logits, softmax and accumulation are fp32; P is rounded to bf16 for the P V product, l sums the
// unrounded fp32 P, as in attn_kernel.
#pragma once
#include "attention.cuh"

namespace p5 {

struct AttnTcCfg {
  static constexpr int HD = 256, ROWS = 128, KT = 64, NS = 4;
  static constexpr int Q_ATOM = ROWS * 128;      // one 64-column block of Q: 16 KB
  static constexpr int Q_BYTES = 4 * Q_ATOM;     // 64 KB
  static constexpr int BOX = KT * 128;           // one 64-column block of a K/V tile: 8 KB
  static constexpr int SLOT = 4 * BOX;           // a K or V tile: 32 KB
  static constexpr int P_BYTES = ROWS * KT * 2;  // 16 KB
  static constexpr int TMEM_COLS = 512;          // S[2] at columns 0 and 64, O at 128..383
  static constexpr int O_COL = 128;
  static constexpr int BAR_OFF = Q_BYTES + NS * SLOT + 2 * P_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr float RESCALE_LOG2 = 8.0f;
  // split-partial staging rows (fp32, 1 KB + 16 B pitch: eight consecutive rows hit distinct 16-byte
  // bank groups), over the Q and K/V ring buffers once every MMA is done
  static constexpr int STG_PITCH = HD * 4 + 16;
  static_assert(ROWS * STG_PITCH <= Q_BYTES + NS * SLOT, "staging must fit in the Q and ring buffers");
};

// One 128-row block (rb) of one batch item / key split (z) with 384 threads: warp 0 loads, warp 1
// issues the MMAs, warps 4-11 run the softmax.  `smem` is 1024-byte aligned with AttnTcCfg::SMEM - 1024
// bytes; tmem_base holds 512 allocated columns.  The tensor maps may live in parameter or global memory.
// Every thread of the CTA calls it; it returns after a CTA-wide barrier with all its MMAs complete.
__device__ __forceinline__ void attn_tc_body(const AttnArgs& a, const CUtensorMap* tq, const CUtensorMap* tk1,
                                             const CUtensorMap* tv1, const CUtensorMap* tk2, const CUtensorMap* tv2,
                                             int* status, uint8_t* smem, uint32_t tmem_base, int rb, int z) {
  using C = AttnTcCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  uint8_t* sQ = smem;
  uint8_t* ring = sQ + C::Q_BYTES;
  uint8_t* sP = ring + C::NS * C::SLOT;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* ring_full = q_full + 1;
  uint64_t* ring_empty = ring_full + C::NS;
  uint64_t* s_full = ring_empty + C::NS;  // [2] S buffer written
  uint64_t* s_empty = s_full + 2;         // [2] S buffer read by all softmax warps
  uint64_t* p_full = s_empty + 2;         // [2] P buffer written (and O rescaled)
  uint64_t* p_empty = p_full + 2;         // [2] P V product done (P buffer free, O updated)
  uint64_t* o_full = p_empty + 2;         // every MMA of the CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = z / a.splits, split = z % a.splits;
  // keys of segment 1 this batch item attends to (a padded prompt's tail is left out): the key tiles past
  // them are skipped, so the item's tile list is [segment-1 tiles with keys | segment-2 tiles]
  const int len1 = a.valid1 ? max(0, min(a.len1, a.valid1[b])) : a.len1;
  const int n1 = (len1 + C::KT - 1) / C::KT, n2 = (a.len2 + C::KT - 1) / C::KT;
  const int tps = a.keys_per_split / C::KT;
  const int t0 = split * tps;
  const int n = max(0, min(n1 + n2, t0 + tps) - t0);  // 0: an empty split (partial m = -inf, l = 0, O = 0)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&ring_full[s], 1);
      mbar_init(&ring_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);  // one arrival per softmax warp
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(o_full, 1);
    flags[0] = 0;
    fence_barrier_init();
    tma_prefetch_desc(tq);
    tma_prefetch_desc(tk1);
    tma_prefetch_desc(tv1);
    tma_prefetch_desc(tk2);
    tma_prefetch_desc(tv2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // tile t of this batch item's key list -> (segment, first key row in it, keys present)
  auto tile_of = [&](int t, int& seg, int& row0, int& valid) {
    seg = t < n1 ? 0 : 1;
    row0 = (seg == 0 ? t : t - n1) * C::KT;
    valid = min(C::KT, (seg == 0 ? len1 : a.len2) - row0);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: Q once, then K_i / V_(i-1) in MMA consumption order
      if (a.pdl) pdl_wait();
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int c = 0; c < 4; ++c) tma_load_4d(sQ + c * C::Q_ATOM, tq, q_full, c * 64, 0, rb * 16, b);
      int it = 0;
      for (int i = 0; i <= n && !flags[0]; ++i) {
        for (int kind = 0; kind < 2; ++kind) {
          if ((kind == 0 && i >= n) || (kind == 1 && i == 0)) continue;
          int seg, row0, valid;
          tile_of(t0 + (kind == 0 ? i : i - 1), seg, row0, valid);
          const int s = it % C::NS;
          const uint32_t ph = (uint32_t)(it / C::NS) & 1u;
          if (!mbar_wait(&ring_empty[s], ph ^ 1u, status, P5_ERR_WAIT_ATTN)) {
            flags[0] = 1;
            break;
          }
          const CUtensorMap* m = kind == 0 ? (seg == 0 ? tk1 : tk2) : (seg == 0 ? tv1 : tv2);
          mbar_arrive_expect_tx(&ring_full[s], C::SLOT);
          for (int c = 0; c < 4; ++c) tma_load_3d(ring + s * C::SLOT + c * C::BOX, m, &ring_full[s], c * 64, row0, b);
          ++it;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::KT);
      constexpr uint32_t idesc_o = mma_idesc_bf16(128, C::HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), ring_addr = smem_u32(ring), p_addr = smem_u32(sP);
      if (!mbar_wait(q_full, 0, status, P5_ERR_WAIT_ATTN)) flags[0] = 1;
      tc_fence_after();
      int it = 0;
      for (int i = 0; i <= n && !flags[0]; ++i) {
        if (i < n) {
          const int s = it % C::NS, sb = i & 1;
          if (!mbar_wait(&ring_full[s], (uint32_t)(it / C::NS) & 1u, status, P5_ERR_WAIT_ATTN) ||
              !mbar_wait(&s_empty[sb], ((uint32_t)(i >> 1) & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = ring_addr + s * C::SLOT;
#pragma unroll
          for (int kk = 0; kk < C::HD / 16; ++kk)
            tc_mma_f16(tmem_base + (uint32_t)(sb * C::KT),
                       sw128_kmajor_desc(q_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                       sw128_kmajor_desc(k_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
          tc_commit(&ring_empty[s]);
          tc_commit(&s_full[sb]);
          ++it;
        }
        if (i >= 1) {
          const int j = i - 1, pb = j & 1;
          const int s = it % C::NS;
          if (!mbar_wait(&ring_full[s], (uint32_t)(it / C::NS) & 1u, status, P5_ERR_WAIT_ATTN) ||
              !mbar_wait(&p_full[pb], (uint32_t)(j >> 1) & 1u, status, P5_ERR_WAIT_ATTN)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = ring_addr + s * C::SLOT;
#pragma unroll
          for (int kk = 0; kk < C::KT / 16; ++kk)
            tc_mma_f16(tmem_base + C::O_COL, sw128_kmajor_desc(p_addr + pb * C::P_BYTES + kk * 32),
                       sw128_mnmajor_desc(v_addr + kk * 2048, C::BOX), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&ring_empty[s]);
          tc_commit(&p_empty[pb]);
          ++it;
        }
      }
      tc_commit(o_full);  // all MMAs issued above are complete (or the pipeline was abandoned)
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- softmax: two warpgroups; thread = query row = TMEM lane, warpgroup g
    // exponentiates S columns [32g, 32g+32) and owns O columns [128g, 128g+128).  Both compute the
    // row max over all 64 columns, so they agree on the running max without exchanging it.
    const int g = (warp - 4) >> 2, sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(sub * 32) << 16);
    const uint32_t t_o = t_lane + (uint32_t)(C::O_COL + g * (C::HD / 2));
    uint8_t* prow = sP + r * 128;
    // two prefix attention groups: this row's query token sees segment-1 keys below group1 only
    const int qtok = (rb * C::ROWS + r) / a.G;
    const int glim = (a.group1 > 0 && qtok < a.group1) ? a.group1 : 0x7fffffff;
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      bool ok = !flags[0] && mbar_wait(&s_full[sb], (uint32_t)(j >> 1) & 1u, status, P5_ERR_WAIT_ATTN);
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t ra[32], rc[32];
      tmem_ld32(t_lane + (uint32_t)(sb * C::KT), ra);
      tmem_ld32(t_lane + (uint32_t)(sb * C::KT + 32), rc);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);

      int seg, row0, valid;
      tile_of(t0 + j, seg, row0, valid);
      if (seg == 0) valid = min(valid, glim - row0);  // may be <= 0: every key of the tile masked for this row
      if (valid < C::KT) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c >= valid) ra[c] = __float_as_uint(-INFINITY);
          if (c + 32 >= valid) rc[c] = __float_as_uint(-INFINITY);
        }
      }
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmaxf(__uint_as_float(ra[k]), __uint_as_float(rc[k]));
#pragma unroll
      for (int c = 8; c < 32; c += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmax3(mx[k], __uint_as_float(ra[c + k]), __uint_as_float(rc[c + k]));
      const float mt = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], fmax3(mx[5], mx[6], mx[7])));
      bool need = false;
      float alpha = 1.f;
      if (j == 0) {
        m_run = mt;
      } else if ((mt - m_run) * LOG2E > C::RESCALE_LOG2) {
        need = true;
        alpha = ex2_approx((m_run - mt) * LOG2E);
        m_run = mt;
        l_run *= alpha;
      }
      // a row with no key yet (m_run = -inf: masked tiles at the start of a key split) gets p = 0
      const float msc = m_run == -INFINITY ? 0.f : m_run * LOG2E;
      uint32_t pk[16];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float s0 = __uint_as_float(g ? rc[2 * c] : ra[2 * c]);
        const float s1 = __uint_as_float(g ? rc[2 * c + 1] : ra[2 * c + 1]);
        const float p0 = ex2_approx(fmaf(s0, LOG2E, -msc));
        const float p1 = ex2_approx(fmaf(s1, LOG2E, -msc));
        ls[c & 3] += p0 + p1;
        pk[c] = pack_bf2(p0, p1);
      }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // P buffer sb was last read by the P V product of tile j-2
      ok = mbar_wait(&p_empty[sb], ((uint32_t)(j >> 1) & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN);
      uint8_t* pdst = prow + sb * C::P_BYTES;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(pdst + (((4 * g + c) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      if (__any_sync(0xffffffffu, need)) {
        // the running max moved: wait for the P V product of tile j-1, then rescale this warp's O part
        ok = ok && mbar_wait(&p_empty[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, status, P5_ERR_WAIT_ATTN);
        if (__any_sync(0xffffffffu, !ok)) {
          flags[0] = 1;
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < C::HD / 2; c += 32) {
          uint32_t o[32];
          tmem_ld32(t_o + (uint32_t)c, o);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st32(t_o + (uint32_t)c, o);
        }
        tmem_wait_st();
      } else if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }

    // ---------------- epilogue: O / l (or the split partials) straight from TMEM
    const bool done = mbar_wait(o_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    // l = the two warpgroups' partial sums, added in a fixed order (P buffers are free: every MMA is done)
    float* lx = reinterpret_cast<float*>(sP);
    lx[g * C::ROWS + r] = l_run;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l_tot = lx[r] + lx[C::ROWS + r];
    if (a.pdl) pdl_wait();
    const int rows_total = a.T * 8;
    const int row = rb * C::ROWS + r;
    // an empty split stores its neutral partial (the merge gives it weight 0); otherwise n > 0
    const bool empty = n == 0 && a.splits > 1;
    const bool store = __all_sync(0xffffffffu, done && alive && (n > 0 || empty)) && row < rows_total;
    const int tok = row >> 3, hq = row & 7;
    const float inv = l_tot > 0.f ? 1.0f / l_tot : 0.f;
    const long base = (long)z * rows_total + row;
#pragma unroll 1
    for (int c = 0; c < C::HD / 2; c += 32) {
      uint32_t o[32];
      __syncwarp();
      tmem_ld32(t_o + (uint32_t)c, o);
      tmem_wait_ld();
      if (empty) {  // no MMA wrote this accumulator
#pragma unroll
        for (int k = 0; k < 32; ++k) o[k] = 0u;
      }
      const int col = g * (C::HD / 2) + c;
      if (!store) {
      } else if (a.splits == 1) {
        // the normalised bf16 row, staged like the split partials and written out by row below
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + col * 2);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf2(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                              pack_bf2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                              pack_bf2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                              pack_bf2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
      } else if (a.ws_half) {
        // split partial O / l in fp16 (half the bytes to drain from this SM), staged like the bf16 rows
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + col * 2);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_h2_sat(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                              pack_h2_sat(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                              pack_h2_sat(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                              pack_h2_sat(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
      } else {
        // split partial: staged in the (now idle) Q / K / V buffers, written out by row below
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + col * 4);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
    }
    {
      // one bulk copy per row (512 B of bf16 output or fp16 split partial, or the 1 KB fp32 one): a thread's own
      // row is far from its lane neighbours', so direct stores would be 32 segments per warp instruction
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 256;" ::: "memory");  // both warpgroups' halves of every row are staged
      if (store && g == 0) {
        if (a.splits == 1)
          bulk_store_global(a.out + b * a.o_bstride + (long)tok * a.ldo + hq * C::HD, smem_u32(smem + r * C::STG_PITCH),
                            C::HD * 2);
        else if (a.ws_half)
          bulk_store_global(reinterpret_cast<__half*>(a.ws_o) + base * C::HD, smem_u32(smem + r * C::STG_PITCH),
                            C::HD * 2);
        else
          bulk_store_global(a.ws_o + base * C::HD, smem_u32(smem + r * C::STG_PITCH), C::HD * 4);
        bulk_store_wait_read();  // the staging buffer must outlive the copy's reads
      }
    }
    if (store && g == 0) {
      if (a.splits == 1) {
        if (a.lse) a.lse[b * a.lse_b + row] = m_run + logf(l_tot);
      } else {
        a.ws_ml[base * 2] = m_run;
        a.ws_ml[base * 2 + 1] = l_tot;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

__global__ void __launch_bounds__(384, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk1,
                   const __grid_constant__ CUtensorMap tv1, const __grid_constant__ CUtensorMap tk2,
                   const __grid_constant__ CUtensorMap tv2, const AttnArgs a, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  __shared__ uint32_t tmem_slot;
  __shared__ int skip;
  // a device-side wait already gave up in an earlier kernel: skip the work (uniformly for the CTA)
  if (threadIdx.x == 0) skip = status ? *((volatile int*)status) : 0;
  __syncthreads();
  if (skip != 0) return;
  if ((threadIdx.x >> 5) == 2) {
    tmem_alloc(&tmem_slot, AttnTcCfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  if (a.pdl) pdl_launch_dependents();
  attn_tc_body(a, &tq, &tk1, &tv1, &tk2, &tv2, status, smem, tmem_base, blockIdx.x, blockIdx.z);
  if ((threadIdx.x >> 5) == 2) tmem_dealloc(tmem_base, AttnTcCfg::TMEM_COLS);
}

}  // namespace p5

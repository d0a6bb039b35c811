// attention_bwd_tc.cuh — dQ of the MQA attention backward on the 5th-generation tensor cores.
//
// Same contract as attn_bwd_dq_kernel (attention_bwd.cuh): for the folded query rows (token, head) of
// one batch item, with P = exp(S - LSE), S = q k^T (q already scaled by 1/16), dP = dO v^T and
// D[row] = sum_d dO*O:  dS = P * (dP - D),  dQ = dS K  over the keys [segment 1 || segment 2].
// Built like attn_tc_kernel:
//   * a CTA owns 128 query rows; Q and dO (128 x 256 bf16 each) stay in 128-byte-swizzled K-major
//     shared memory, loaded once by 4-D TMA boxes;
//   * key tiles of 64 (never straddling the two segments) arrive by 3-D TMA into one K slot and one
//     V slot; one thread issues S = Q K^T and dP = dO V^T (M=128, N=64, K=256) into TMEM and, once the
//     elementwise warps have written dS (bf16, K-major) to shared memory, dQ += dS K (N=256, K read
//     MN-major straight from its [key][dim] layout) into a 256-column TMEM accumulator;
//   * eight elementwise warps: thread = query row = TMEM lane, warpgroup g takes key columns
//     [32g, 32g+32) of the tile; P uses exp2f as attn_bwd_dq_kernel does, dS is rounded to bf16 for
//     the MMA (as that kernel's mma.sync A fragments are);
//   * the V slot is refilled as soon as dP is done, the K slot once dQ has consumed it.
// dQ rows are staged in the idle Q / dO buffers and written by one 512-byte bulk copy per row.
#pragma once
#include "attention_bwd.cuh"

namespace p5 {

struct AttnBwdTcCfg {
  static constexpr int HD = 256, ROWS = 128, KT = 64;
  static constexpr int Q_ATOM = ROWS * 128;      // one 64-column block of a 128-row tile: 16 KB
  static constexpr int Q_BYTES = 4 * Q_ATOM;     // 64 KB
  static constexpr int BOX = KT * 128;           // one 64-column block of a key tile: 8 KB
  static constexpr int SLOT = 4 * BOX;           // a K or V tile: 32 KB
  static constexpr int E_BYTES = ROWS * KT * 2;  // dS tile, bf16: 16 KB
  static constexpr int O_OFF = Q_BYTES, K_OFF = 2 * Q_BYTES, V_OFF = K_OFF + SLOT, E_OFF = V_OFF + SLOT;
  static constexpr int BAR_OFF = E_OFF + E_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr uint32_t TMEM_COLS = 512;     // S at 0, dP at 64, dQ at 128..383
  static constexpr int DP_COL = 64, ACC_COL = 128;
  static constexpr int STG_PITCH = HD * 2 + 16;  // bf16 output rows, 16 bytes of skew
  static_assert(ROWS * STG_PITCH <= 2 * Q_BYTES, "output staging must fit in the Q and dO buffers");
};

// grid (query-row blocks of 128, 1, batch), 384 threads: warp 0 loads, warp 1 issues the MMAs, warp 2
// owns TMEM, warps 4-11 compute dS and write dQ.  Every wait is bounded and records P5_ERR_WAIT_ATTN.
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                          const __grid_constant__ CUtensorMap tk1, const __grid_constant__ CUtensorMap tv1,
                          const __grid_constant__ CUtensorMap tk2, const __grid_constant__ CUtensorMap tv2,
                          const AttnBwdArgs a, int* status) {
  using C = AttnBwdTcCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sO = smem + C::O_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sE = smem + C::E_OFF;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = q_full + 2;
  uint64_t* v_full = q_full + 3;
  uint64_t* v_empty = q_full + 4;
  uint64_t* sd_full = q_full + 5;   // S and dP of the tile in TMEM
  uint64_t* sd_empty = q_full + 6;  // read by all eight elementwise warps
  uint64_t* e_full = q_full + 7;    // dS written by all eight elementwise warps
  uint64_t* e_empty = q_full + 8;   // dQ MMA done with dS (and with the K slot)
  uint64_t* o_full = q_full + 9;    // every MMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 10);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] skip

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, b = blockIdx.z;
  const QSeg& qs = a.qs;
  const int rows = qs.T * P5_NH;
  const int n1 = (a.len1 + C::KT - 1) / C::KT, n2 = (a.len2 + C::KT - 1) / C::KT, n = n1 + n2;
  auto tile_of = [&](int t, int& seg, int& row0, int& valid) {
    seg = t < n1 ? 0 : 1;
    row0 = (seg == 0 ? t : t - n1) * C::KT;
    valid = min(C::KT, (seg == 0 ? a.len1 : a.len2) - row0);
  };

  if (threadIdx.x == 0) flags[1] = status ? *((volatile int*)status) : 0;
  __syncthreads();
  if (flags[1] != 0) return;  // a device-side wait already gave up earlier: skip (uniform for the CTA)
  if (threadIdx.x == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(q_full + i, (i == 6 || i == 7) ? 8 : 1);
    flags[0] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
    tma_prefetch_desc(&tk1);
    tma_prefetch_desc(&tv1);
    tma_prefetch_desc(&tk2);
    tma_prefetch_desc(&tv2);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: Q and dO once; per tile V then K (V frees first)
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(sQ + c * C::Q_ATOM, &tq, q_full, c * 64, 0, rb * 16, b);
        tma_load_4d(sO + c * C::Q_ATOM, &tdo, q_full, c * 64, 0, rb * 16, b);
      }
      for (int j = 0; j < n && !flags[0]; ++j) {
        int seg, row0, valid;
        tile_of(j, seg, row0, valid);
        const uint32_t ph = ((uint32_t)j & 1u) ^ 1u;
        if (!mbar_wait(v_empty, ph, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(v_full, C::SLOT);
        for (int c = 0; c < 4; ++c) tma_load_3d(sV + c * C::BOX, seg == 0 ? &tv1 : &tv2, v_full, c * 64, row0, b);
        if (!mbar_wait(k_empty, ph, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(k_full, C::SLOT);
        for (int c = 0; c < 4; ++c) tma_load_3d(sK + c * C::BOX, seg == 0 ? &tk1 : &tk2, k_full, c * 64, row0, b);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::KT);
      constexpr uint32_t idesc_o = mma_idesc_bf16(128, C::HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), o_addr = smem_u32(sO), k_addr = smem_u32(sK), v_addr = smem_u32(sV),
                     e_addr = smem_u32(sE);
      if (!mbar_wait(q_full, 0, status, P5_ERR_WAIT_ATTN)) flags[0] = 1;
      tc_fence_after();
      for (int j = 0; j < n && !flags[0]; ++j) {
        const uint32_t ph = (uint32_t)j & 1u;
        if (!mbar_wait(k_full, ph, status, P5_ERR_WAIT_ATTN) ||
            !mbar_wait(sd_empty, ph ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(q_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(k_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        if (!mbar_wait(v_full, ph, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(tmem_base + C::DP_COL, sw128_kmajor_desc(o_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(v_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(v_empty);
        tc_commit(sd_full);
        if (!mbar_wait(e_full, ph, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::KT / 16; ++kk)
          tc_mma_f16(tmem_base + C::ACC_COL, sw128_kmajor_desc(e_addr + kk * 32),
                     sw128_mnmajor_desc(k_addr + kk * 2048, C::BOX), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(k_empty);
        tc_commit(e_empty);
      }
      tc_commit(o_full);  // all MMAs issued above are complete (or the pipeline was abandoned)
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- dS: thread = query row = TMEM lane, warpgroup g takes key columns [32g, 32g+32)
    const int g = (warp - 4) >> 2, sub = warp & 3;
    const int r = sub * 32 + lane, row = rb * C::ROWS + r;
    const bool vrow = row < rows;
    const float lse = vrow ? qs.lse[b * qs.lb + row] : 1e30f;
    const float dd = vrow ? qs.Dv[b * qs.lb + row] : 0.f;
    const uint32_t t_lane = tmem_base + ((uint32_t)(sub * 32) << 16);
    uint8_t* erow = sE + r * 128;
    bool alive = true;
    for (int j = 0; j < n; ++j) {
      const uint32_t ph = (uint32_t)j & 1u;
      bool ok = !flags[0] && mbar_wait(sd_full, ph, status, P5_ERR_WAIT_ATTN);
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t rs[32], rp[32];
      tmem_ld32(t_lane + (uint32_t)(32 * g), rs);
      tmem_ld32(t_lane + (uint32_t)(C::DP_COL + 32 * g), rp);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sd_empty);
      int seg, row0, valid;
      tile_of(j, seg, row0, valid);
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float e2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = 32 * g + 2 * c + h;
          const float p = col < valid ? exp2f((__uint_as_float(rs[2 * c + h]) - lse) * LOG2E) : 0.f;
          e2[h] = p * (__uint_as_float(rp[2 * c + h]) - dd);
        }
        pk[c] = pack_bf2(e2[0], e2[1]);
      }
      ok = mbar_wait(e_empty, ph ^ 1u, status, P5_ERR_WAIT_ATTN);  // the dQ MMA of tile j-1 read dS
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(erow + (((4 * g + c) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(e_full);
    }

    // ---------------- dQ: TMEM -> bf16 rows staged over Q / dO -> one bulk copy per row
    const bool done = mbar_wait(o_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    const bool store = __all_sync(0xffffffffu, done && alive && n > 0) && vrow;
#pragma unroll 1
    for (int c = 0; c < C::HD / 2; c += 32) {
      uint32_t o[32];
      __syncwarp();
      tmem_ld32(t_lane + (uint32_t)(C::ACC_COL + g * (C::HD / 2) + c), o);
      tmem_wait_ld();
      if (store) {
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + (g * (C::HD / 2) + c) * 2);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf2(__uint_as_float(o[8 * q]), __uint_as_float(o[8 * q + 1])),
                              pack_bf2(__uint_as_float(o[8 * q + 2]), __uint_as_float(o[8 * q + 3])),
                              pack_bf2(__uint_as_float(o[8 * q + 4]), __uint_as_float(o[8 * q + 5])),
                              pack_bf2(__uint_as_float(o[8 * q + 6]), __uint_as_float(o[8 * q + 7])));
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 256;" ::: "memory");  // both halves of every row are staged
    if (store && g == 0) {
      bf16* dst = a.dq + b * a.dq_b + (long)(row / 8) * a.ld_dq + (row % 8) * C::HD;
      bulk_store_global(dst, smem_u32(smem + r * C::STG_PITCH), C::HD * 2);
      bulk_store_wait_read();  // the staging buffer must outlive the copy's reads
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

namespace p5 {

// ---------------------------------------------------------------- dK / dV on tcgen05
// dK = dS^T Q, dV = P^T dO for 128 keys of segment a.kseg per CTA (blockIdx.x), the query rows of the
// segments qa (then qbseg when a.nq == 2) in tiles of 64 rows (8 tokens x 8 heads), tiles
// [y * nt / gridDim.y, (y + 1) * nt / gridDim.y) for y = blockIdx.y.  The keys (and V for dK) stay
// resident; S^T = K Q^T and dP^T = V dO^T (M=128 keys, N=64 rows) go to TMEM; the elementwise warps
// (thread = key) form P^T = exp(S^T - LSE[col]) and dS^T = P^T (dP^T - D[col]) in bf16 K-major shared
// memory; the accumulate reads Q (dK) or dO (dV) MN-major.  With one query split the bf16 rows go to
// out; with several, fp32 partial rows go to ws[((b * gridDim.x + x) * gridDim.y + y) * 128 + key]
// and attn_bwd_dkv_reduce_kernel sums them in split order.
constexpr int ABW_KV_MAX_SPLITS = 8;  // query-split partials the trainer's workspace holds

struct AttnBwdKvCfg {
  static constexpr int HD = 256, KEYS = 128, QT = 64;
  static constexpr int R_ATOM = KEYS * 128;      // one 64-dim block of the 128 resident keys: 16 KB
  static constexpr int R_BYTES = 4 * R_ATOM;     // 64 KB
  static constexpr int BOX = QT * 128;           // one 64-dim block of a 64-row query tile: 8 KB
  static constexpr int SLOT = 4 * BOX;           // 32 KB
  static constexpr int E_BYTES = KEYS * QT * 2;  // 16 KB
  static constexpr int V_OFF = R_BYTES, A_OFF = 2 * R_BYTES, B_OFF = A_OFF + SLOT, E_OFF = B_OFF + SLOT;
  static constexpr int BAR_OFF = E_OFF + E_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr uint32_t TMEM_COLS = 512;     // S^T at 0, dP^T at 64, accumulator at 128..383
  static constexpr int DP_COL = 64, ACC_COL = 128;
  static constexpr int STG_PITCH = HD * 4 + 16;  // fp32 rows (or bf16 rows in the first half)
  static_assert(KEYS * STG_PITCH <= B_OFF, "staging must fit in the resident and first slot buffers");
};

template <bool DK>
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                           const __grid_constant__ CUtensorMap tqa, const __grid_constant__ CUtensorMap tdoa,
                           const __grid_constant__ CUtensorMap tqb, const __grid_constant__ CUtensorMap tdob,
                           const AttnBwdArgs a, float* ws, int* status) {
  using C = AttnBwdKvCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sK = smem;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sA = smem + C::A_OFF;  // Q tile
  uint8_t* sB = smem + C::B_OFF;  // dO tile
  uint8_t* sE = smem + C::E_OFF;
  uint64_t* r_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* a_full = r_full + 1;
  uint64_t* a_empty = r_full + 2;
  uint64_t* b_full = r_full + 3;
  uint64_t* b_empty = r_full + 4;
  uint64_t* sd_full = r_full + 5;
  uint64_t* sd_empty = r_full + 6;  // 8 arrivals
  uint64_t* e_full = r_full + 7;    // 8 arrivals
  uint64_t* e_empty = r_full + 8;
  uint64_t* o_full = r_full + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(r_full + 10);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.x, y = blockIdx.y, b = blockIdx.z;
  const int seg_len = a.kseg == 1 ? a.len1 : a.len2;
  const int k0 = kb * C::KEYS;
  const int na = (a.qa.T + 7) / 8, nbq = a.nq > 1 ? (a.qbseg.T + 7) / 8 : 0, nt = na + nbq;
  const int j0 = (int)((long)y * nt / gridDim.y), j1 = (int)((long)(y + 1) * nt / gridDim.y), n = j1 - j0;
  // query tile j: segment (0 = qa, 1 = qbseg) and first token
  auto tile_of = [&](int j, int& sg, int& tok0) {
    sg = j < na ? 0 : 1;
    tok0 = (sg == 0 ? j : j - na) * 8;
  };

  if (threadIdx.x == 0) flags[1] = status ? *((volatile int*)status) : 0;
  __syncthreads();
  if (flags[1] != 0) return;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(r_full + i, (i == 6 || i == 7) ? 8 : 1);
    flags[0] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tk);
    if (DK) tma_prefetch_desc(&tv);
    tma_prefetch_desc(&tqa);
    tma_prefetch_desc(&tdoa);
    tma_prefetch_desc(&tqb);
    tma_prefetch_desc(&tdob);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: keys (and V) once; per query tile the slot that frees first
      // (dO for dK, after dP^T; Q for dV, after S^T) is refilled first
      mbar_arrive_expect_tx(r_full, (DK ? 2 : 1) * C::R_BYTES);
      for (int c = 0; c < 4; ++c) {
        tma_load_3d(sK + c * C::R_ATOM, &tk, r_full, c * 64, k0, b);
        if (DK) tma_load_3d(sV + c * C::R_ATOM, &tv, r_full, c * 64, k0, b);
      }
      for (int i = 0; i < n && !flags[0]; ++i) {
        int sg, tok0;
        tile_of(j0 + i, sg, tok0);
        const uint32_t ph = ((uint32_t)i & 1u) ^ 1u;
        for (int w = 0; w < 2; ++w) {
          const bool q_slot = DK ? (w == 1) : (w == 0);
          uint64_t* emp = q_slot ? a_empty : b_empty;
          uint64_t* ful = q_slot ? a_full : b_full;
          uint8_t* dst = q_slot ? sA : sB;
          const CUtensorMap* m = q_slot ? (sg == 0 ? &tqa : &tqb) : (sg == 0 ? &tdoa : &tdob);
          if (!mbar_wait(emp, ph, status, P5_ERR_WAIT_ATTN)) {
            flags[0] = 1;
            break;
          }
          mbar_arrive_expect_tx(ful, C::SLOT);
          for (int c = 0; c < 4; ++c) tma_load_4d(dst + c * C::BOX, m, ful, c * 64, 0, tok0, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::QT);
      constexpr uint32_t idesc_o = mma_idesc_bf16(128, C::HD, false, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), qa_addr = smem_u32(sA), ob_addr = smem_u32(sB),
                     e_addr = smem_u32(sE);
      if (!mbar_wait(r_full, 0, status, P5_ERR_WAIT_ATTN)) flags[0] = 1;
      tc_fence_after();
      for (int i = 0; i < n && !flags[0]; ++i) {
        const uint32_t ph = (uint32_t)i & 1u;
        if (!mbar_wait(a_full, ph, status, P5_ERR_WAIT_ATTN) ||
            !mbar_wait(sd_empty, ph ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(k_addr + (kk >> 2) * C::R_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(qa_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        if (DK) {
          if (!mbar_wait(b_full, ph, status, P5_ERR_WAIT_ATTN)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C::HD / 16; ++kk)
            tc_mma_f16(tmem_base + C::DP_COL, sw128_kmajor_desc(v_addr + (kk >> 2) * C::R_ATOM + (kk & 3) * 32),
                       sw128_kmajor_desc(ob_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
          tc_commit(b_empty);
        } else {
          tc_commit(a_empty);
        }
        tc_commit(sd_full);
        if (!mbar_wait(e_full, ph, status, P5_ERR_WAIT_ATTN) ||
            (!DK && !mbar_wait(b_full, ph, status, P5_ERR_WAIT_ATTN))) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc_b = DK ? qa_addr : ob_addr;
#pragma unroll
        for (int kk = 0; kk < C::QT / 16; ++kk)
          tc_mma_f16(tmem_base + C::ACC_COL, sw128_kmajor_desc(e_addr + kk * 32),
                     sw128_mnmajor_desc(acc_b + kk * 2048, C::BOX), idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(DK ? a_empty : b_empty);
        tc_commit(e_empty);
      }
      tc_commit(o_full);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- P^T / dS^T: thread = key = TMEM lane, warpgroup g takes query columns [32g, 32g+32)
    const int g = (warp - 4) >> 2, sub = warp & 3;
    const int r = sub * 32 + lane, key = k0 + r;
    const uint32_t t_lane = tmem_base + ((uint32_t)(sub * 32) << 16);
    uint8_t* erow = sE + r * 128;
    bool alive = true;
    for (int i = 0; i < n; ++i) {
      const uint32_t ph = (uint32_t)i & 1u;
      int sg, tok0;
      tile_of(j0 + i, sg, tok0);
      const QSeg& qs = sg == 0 ? a.qa : a.qbseg;
      const int rows = qs.T * P5_NH, rbase = tok0 * P5_NH + 32 * g;
      // the 32 columns' LSE and D (the same for every thread of the warpgroup); rows past the
      // segment read its last row and are masked below
      float lse[32], dd[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const long ix = b * qs.lb + min(rbase + c, rows - 1);
        lse[c] = qs.lse[ix];
        dd[c] = DK ? qs.Dv[ix] : 0.f;
      }
      bool ok = !flags[0] && mbar_wait(sd_full, ph, status, P5_ERR_WAIT_ATTN);
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t rs[32], rp[32];
      tmem_ld32(t_lane + (uint32_t)(32 * g), rs);
      if (DK) tmem_ld32(t_lane + (uint32_t)(C::DP_COL + 32 * g), rp);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sd_empty);
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float e2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int cc = 2 * c + h;
          const float p = rbase + cc < rows ? exp2f((__uint_as_float(rs[cc]) - lse[cc]) * LOG2E) : 0.f;
          e2[h] = DK ? p * (__uint_as_float(rp[cc]) - dd[cc]) : p;
        }
        pk[c] = pack_bf2(e2[0], e2[1]);
      }
      ok = mbar_wait(e_empty, ph ^ 1u, status, P5_ERR_WAIT_ATTN);  // the accumulate of tile i-1 read it
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(erow + (((4 * g + c) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(e_full);
    }

    // ---------------- accumulator -> rows staged over the resident buffers -> one bulk copy per row
    const bool done = mbar_wait(o_full, 0, status, P5_ERR_WAIT_ATTN);
    tc_fence_after();
    const bool store = __all_sync(0xffffffffu, done && alive) && key < seg_len;
    const bool part = gridDim.y > 1;
#pragma unroll 1
    for (int c = 0; c < C::HD / 2; c += 32) {
      uint32_t o[32];
      __syncwarp();
      tmem_ld32(t_lane + (uint32_t)(C::ACC_COL + g * (C::HD / 2) + c), o);
      tmem_wait_ld();
      if (!n) {
#pragma unroll
        for (int q = 0; q < 32; ++q) o[q] = 0u;  // an empty split contributes zeros
      }
      const int col = g * (C::HD / 2) + c;
      if (store && part) {
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + col * 4);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      } else if (store) {
        uint4* dst = reinterpret_cast<uint4*>(smem + r * C::STG_PITCH + col * 2);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf2(__uint_as_float(o[8 * q]), __uint_as_float(o[8 * q + 1])),
                              pack_bf2(__uint_as_float(o[8 * q + 2]), __uint_as_float(o[8 * q + 3])),
                              pack_bf2(__uint_as_float(o[8 * q + 4]), __uint_as_float(o[8 * q + 5])),
                              pack_bf2(__uint_as_float(o[8 * q + 6]), __uint_as_float(o[8 * q + 7])));
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (store && g == 0) {
      if (part) {
        float* dst = ws + ((((long)b * gridDim.x + kb) * gridDim.y + y) * C::KEYS + r) * C::HD;
        bulk_store_global(dst, smem_u32(smem + r * C::STG_PITCH), C::HD * 4);
      } else {
        bf16* dst = (DK ? a.dk : a.dv) + b * a.dkv_b + (long)key * a.ld_dkv;
        bulk_store_global(dst, smem_u32(smem + r * C::STG_PITCH), C::HD * 2);
      }
      bulk_store_wait_read();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Sum of the query-split partials of attn_bwd_dkv_tc_kernel in split order: out[b][key][d] (bf16),
// 8 dims per thread.
__global__ void attn_bwd_dkv_reduce_kernel(const float* ws, int kblocks, int splits, int seg_len, int nb, bf16* out,
                                           int ld, long bstride) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)nb * seg_len * 32) return;
  const int d8 = (int)(i % 32), key = (int)((i / 32) % seg_len), b = (int)(i / 32 / seg_len);
  const int kb = key / AttnBwdKvCfg::KEYS, r = key % AttnBwdKvCfg::KEYS;
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int y = 0; y < splits; ++y) {
    const float4* src = reinterpret_cast<const float4*>(
        ws + ((((long)b * kblocks + kb) * splits + y) * AttnBwdKvCfg::KEYS + r) * AttnBwdKvCfg::HD + d8 * 8);
    const float4 u = src[0], v = src[1];
    s[0] += u.x;
    s[1] += u.y;
    s[2] += u.z;
    s[3] += u.w;
    s[4] += v.x;
    s[5] += v.y;
    s[6] += v.z;
    s[7] += v.w;
  }
  *reinterpret_cast<uint4*>(out + b * bstride + (long)key * ld + d8 * 8) =
      make_uint4(pack_bf2(s[0], s[1]), pack_bf2(s[2], s[3]), pack_bf2(s[4], s[5]), pack_bf2(s[6], s[7]));
}

}  // namespace p5

// attention_bwd_dq_pipe.cuh — dQ of the MQA attention backward on tcgen05 with the dS step overlapped.
//
// Same contract and arithmetic as attn_bwd_dq_tc_kernel (attention_bwd_tc.cuh): for 128 folded query
// rows (token, head) of one batch item, P = exp(S - LSE) with S = q k^T, dP = dO v^T,
// dS = P * (dP - D), dQ = sum over the 64-key tiles of dS K, keys [segment 1 || segment 2].
// The schedule differs: S and dP of tile j+1 are issued before the dQ update of tile j, into the other
// of two TMEM buffer pairs, so the tensor core computes tile j+1 while the elementwise warps form dS of
// tile j (in the one-slot kernel they ran one after the other: 30 % of the issuing thread's time went
// to waiting for dS, measured).  That needs K of tile j+1 while tile j's update still reads K of tile
// j, so K gets two slots; the room comes from keeping dS in tensor memory (bf16, two per 32-bit
// column, written over the S columns the same warpgroup has just read) as the A operand of the dQ
// update, instead of a shared-memory buffer.
// Shared memory: Q and dO (64 KB each, resident), K slots 2 x 32 KB, one V slot (32 KB).
// TMEM columns: buffer b = 0, 1: S at 128b, dP at 128b + 64; dS of warpgroup g at 128b + 32g (16
// columns); dQ at 256..511.  S of tile j+2 overwrites dS of tile j only after the dQ update that reads
// it, because one thread issues both in that order.  Every wait is bounded (P5_ERR_WAIT_ATTN).
#pragma once
#include "attention_bwd_tc.cuh"

namespace p5 {

struct AttnBwdPipeCfg {
  static constexpr int HD = 256, ROWS = 128, KT = 64;
  static constexpr int Q_ATOM = ROWS * 128;      // one 64-dim block of a 128-row tile: 16 KB
  static constexpr int Q_BYTES = 4 * Q_ATOM;     // 64 KB
  static constexpr int BOX = KT * 128;           // one 64-dim block of a key tile: 8 KB
  static constexpr int SLOT = 4 * BOX;           // a K or V tile: 32 KB
  static constexpr int O_OFF = Q_BYTES, K_OFF = 2 * Q_BYTES, V_OFF = K_OFF + 2 * SLOT;
  static constexpr int BAR_OFF = V_OFF + SLOT;   // 224 KB
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int BUF_COLS = 128, DP_COL = 64, ACC_COL = 256;
  static constexpr int STG_PITCH = HD * 2 + 16;  // bf16 output rows, 16 bytes of skew
  static_assert(ROWS * STG_PITCH <= 2 * Q_BYTES, "output staging must fit in the Q and dO buffers");
  static_assert(SMEM <= 232448, "shared memory per block");
  static_assert(KT == AttnBwdTcCfg::KT, "the key tensor maps are shared with the one-slot kernel");
};

// grid (query-row blocks of 128, 1, batch), 384 threads: warp 0 loads, warp 1 issues the MMAs, warp 2
// owns TMEM, warps 4-11 form dS (thread = query row = TMEM lane, warpgroup g takes key columns
// [32g, 32g+32) of the tile) and write dQ.
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dq_pipe_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                            const __grid_constant__ CUtensorMap tk1, const __grid_constant__ CUtensorMap tv1,
                            const __grid_constant__ CUtensorMap tk2, const __grid_constant__ CUtensorMap tv2,
                            const AttnBwdArgs a, int* status) {
  using C = AttnBwdPipeCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sO = smem + C::O_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* k_full = q_full + 1;   // [2]
  uint64_t* k_empty = k_full + 2;  // [2]
  uint64_t* v_full = k_empty + 2;
  uint64_t* v_empty = v_full + 1;
  uint64_t* sd_full = v_empty + 1;  // [2] S and dP of a tile in TMEM buffer b
  uint64_t* e_full = sd_full + 2;   // [2] dS of buffer b written (8 warp arrivals)
  uint64_t* o_full = e_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
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
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&sd_full[i], 1);
      mbar_init(&e_full[i], 8);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(o_full, 1);
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
      // ---------------- TMA producer: Q and dO once; per tile V (freed by its dP) then K (freed by its dQ)
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(sQ + c * C::Q_ATOM, &tq, q_full, c * 64, 0, rb * 16, b);
        tma_load_4d(sO + c * C::Q_ATOM, &tdo, q_full, c * 64, 0, rb * 16, b);
      }
      for (int j = 0; j < n && !flags[0]; ++j) {
        int seg, row0, valid;
        tile_of(j, seg, row0, valid);
        if (!mbar_wait(v_empty, ((uint32_t)j & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(v_full, C::SLOT);
        for (int c = 0; c < 4; ++c) tma_load_3d(sV + c * C::BOX, seg == 0 ? &tv1 : &tv2, v_full, c * 64, row0, b);
        const int ks = j & 1;
        if (!mbar_wait(&k_empty[ks], ((uint32_t)(j >> 1) & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[ks], C::SLOT);
        for (int c = 0; c < 4; ++c)
          tma_load_3d(sK + ks * C::SLOT + c * C::BOX, seg == 0 ? &tk1 : &tk2, &k_full[ks], c * 64, row0, b);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: S(j+1), dP(j+1) go ahead of dQ += dS(j) K(j)
      constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::KT);
      constexpr uint32_t idesc_o = mma_idesc_bf16(128, C::HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), o_addr = smem_u32(sO), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto issue_sdp = [&](int t) -> bool {
        const int ks = t & 1;
        const uint32_t sb = tmem_base + (uint32_t)(ks * C::BUF_COLS);
        if (!mbar_wait(&k_full[ks], (uint32_t)(t >> 1) & 1u, status, P5_ERR_WAIT_ATTN)) return false;
        tc_fence_after();
        const uint32_t kb = k_addr + ks * C::SLOT;
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(sb, sw128_kmajor_desc(q_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(kb + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        if (!mbar_wait(v_full, (uint32_t)t & 1u, status, P5_ERR_WAIT_ATTN)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(sb + C::DP_COL, sw128_kmajor_desc(o_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(v_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(v_empty);
        tc_commit(&sd_full[ks]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, status, P5_ERR_WAIT_ATTN);
      tc_fence_after();
      if (ok && n > 0) ok = issue_sdp(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n && !issue_sdp(j + 1)) {
          ok = false;
          break;
        }
        const int bf = j & 1;
        if (!mbar_wait(&e_full[bf], (uint32_t)(j >> 1) & 1u, status, P5_ERR_WAIT_ATTN)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = k_addr + bf * C::SLOT, ds = tmem_base + (uint32_t)(bf * C::BUF_COLS);
        // dS of keys [16kk, 16kk+16): warpgroup kk/2's 16 columns at 32 (kk/2), 8 columns per K step
#pragma unroll
        for (int kk = 0; kk < C::KT / 16; ++kk)
          tc_mma_f16_ta(tmem_base + C::ACC_COL, ds + (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8),
                        sw128_mnmajor_desc(kb + kk * 2048, C::BOX), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&k_empty[bf]);
      }
      if (!ok) flags[0] = 1;
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
    bool alive = true;
    for (int j = 0; j < n; ++j) {
      const int bf = j & 1;
      bool ok = !flags[0] && mbar_wait(&sd_full[bf], (uint32_t)(j >> 1) & 1u, status, P5_ERR_WAIT_ATTN);
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = t_lane + (uint32_t)(bf * C::BUF_COLS + 32 * g);
      uint32_t rs[32], rp[32];
      tmem_ld32(sb, rs);
      tmem_ld32(sb + C::DP_COL, rp);
      tmem_wait_ld();
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
      tmem_st16(sb, pk);  // over this warpgroup's own S columns, already read
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&e_full[bf]);
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

// ---------------------------------------------------------------- dK / dV with the same overlap
// Contract and arithmetic of attn_bwd_dkv_tc_kernel<DK>: 128 resident keys per CTA (and V for dK), the
// query tiles [j0, j1) of 64 rows, S^T = K Q^T and (dK) dP^T = V dO^T in TMEM, P^T or dS^T by the
// elementwise warps (thread = key), dK += dS^T Q or dV += P^T dO.  Here S^T (and dP^T) of tile i+1 are
// issued before the accumulate of tile i, into the other TMEM buffer pair; the accumulate's operand X
// (Q for dK, dO for dV) gets two slots, the other operand Y (dO for dK, Q for dV) one; P^T / dS^T stay
// in TMEM over the S^T columns of their warpgroup (the A operand of the accumulate).
// Shared memory: K (and V) 64 KB each, X slots 2 x 32 KB at 128 KB, Y slot 32 KB at 192 KB.
struct AttnBwdKvPipeCfg {
  static constexpr int HD = 256, KEYS = 128, QT = 64;
  static constexpr int R_ATOM = KEYS * 128;      // one 64-dim block of the 128 resident keys: 16 KB
  static constexpr int R_BYTES = 4 * R_ATOM;     // 64 KB
  static constexpr int BOX = QT * 128;           // one 64-dim block of a 64-row query tile: 8 KB
  static constexpr int SLOT = 4 * BOX;           // 32 KB
  static constexpr int V_OFF = R_BYTES, X_OFF = 2 * R_BYTES, Y_OFF = X_OFF + 2 * SLOT;
  static constexpr int BAR_OFF = Y_OFF + SLOT;   // 224 KB
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int BUF_COLS = 128, DP_COL = 64, ACC_COL = 256;
  static constexpr int STG_PITCH = HD * 4 + 16;  // fp32 rows (or bf16 rows in the first half)
  static_assert(KEYS * STG_PITCH <= Y_OFF, "staging must fit below the Y slot");
  static_assert(SMEM <= 232448, "shared memory per block");
  static_assert(KEYS == AttnBwdKvCfg::KEYS && QT == AttnBwdKvCfg::QT, "tensor maps shared with the one-slot kernel");
};

template <bool DK>
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dkv_pipe_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                             const __grid_constant__ CUtensorMap tqa, const __grid_constant__ CUtensorMap tdoa,
                             const __grid_constant__ CUtensorMap tqb, const __grid_constant__ CUtensorMap tdob,
                             const AttnBwdArgs a, float* ws, int* status) {
  using C = AttnBwdKvPipeCfg;
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sK = smem;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sX = smem + C::X_OFF;  // Q (dK) or dO (dV) tiles, two slots
  uint8_t* sY = smem + C::Y_OFF;  // dO (dK) or Q (dV) tile
  uint64_t* r_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* x_full = r_full + 1;   // [2]
  uint64_t* x_empty = x_full + 2;  // [2]
  uint64_t* y_full = x_empty + 2;
  uint64_t* y_empty = y_full + 1;
  uint64_t* sd_full = y_empty + 1;  // [2]
  uint64_t* e_full = sd_full + 2;   // [2], 8 arrivals
  uint64_t* o_full = e_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.x, y = blockIdx.y, b = blockIdx.z;
  const int seg_len = a.kseg == 1 ? a.len1 : a.len2;
  const int k0 = kb * C::KEYS;
  const int na = (a.qa.T + 7) / 8, nbq = a.nq > 1 ? (a.qbseg.T + 7) / 8 : 0, nt = na + nbq;
  const int j0 = (int)((long)y * nt / gridDim.y), j1 = (int)((long)(y + 1) * nt / gridDim.y), n = j1 - j0;
  auto tile_of = [&](int j, int& sg, int& tok0) {
    sg = j < na ? 0 : 1;
    tok0 = (sg == 0 ? j : j - na) * 8;
  };

  if (threadIdx.x == 0) flags[1] = status ? *((volatile int*)status) : 0;
  __syncthreads();
  if (flags[1] != 0) return;
  if (threadIdx.x == 0) {
    mbar_init(r_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
      mbar_init(&sd_full[i], 1);
      mbar_init(&e_full[i], 8);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, 1);
    mbar_init(o_full, 1);
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
      // ---------------- TMA producer: keys (and V) once; per query tile Y (one slot) then X (two slots)
      mbar_arrive_expect_tx(r_full, (DK ? 2 : 1) * C::R_BYTES);
      for (int c = 0; c < 4; ++c) {
        tma_load_3d(sK + c * C::R_ATOM, &tk, r_full, c * 64, k0, b);
        if (DK) tma_load_3d(sV + c * C::R_ATOM, &tv, r_full, c * 64, k0, b);
      }
      for (int i = 0; i < n && !flags[0]; ++i) {
        int sg, tok0;
        tile_of(j0 + i, sg, tok0);
        const CUtensorMap* mq = sg == 0 ? &tqa : &tqb;
        const CUtensorMap* mo = sg == 0 ? &tdoa : &tdob;
        if (!mbar_wait(y_empty, ((uint32_t)i & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(y_full, C::SLOT);
        for (int c = 0; c < 4; ++c) tma_load_4d(sY + c * C::BOX, DK ? mo : mq, y_full, c * 64, 0, tok0, b);
        const int xs = i & 1;
        if (!mbar_wait(&x_empty[xs], ((uint32_t)(i >> 1) & 1u) ^ 1u, status, P5_ERR_WAIT_ATTN)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&x_full[xs], C::SLOT);
        for (int c = 0; c < 4; ++c)
          tma_load_4d(sX + xs * C::SLOT + c * C::BOX, DK ? mq : mo, &x_full[xs], c * 64, 0, tok0, b);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: S^T (and dP^T) of tile i+1 ahead of the accumulate of tile i
      constexpr uint32_t idesc_s = mma_idesc_bf16(128, C::QT);
      constexpr uint32_t idesc_o = mma_idesc_bf16(128, C::HD, false, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), x_addr = smem_u32(sX), y_addr = smem_u32(sY);
      auto issue_s = [&](int t) -> bool {
        const int bt = t & 1;
        const uint32_t sb = tmem_base + (uint32_t)(bt * C::BUF_COLS);
        const uint32_t qb = DK ? x_addr + bt * C::SLOT : y_addr;  // the Q tile
        if (DK) {
          if (!mbar_wait(&x_full[bt], (uint32_t)(t >> 1) & 1u, status, P5_ERR_WAIT_ATTN)) return false;
        } else if (!mbar_wait(y_full, (uint32_t)t & 1u, status, P5_ERR_WAIT_ATTN)) {
          return false;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::HD / 16; ++kk)
          tc_mma_f16(sb, sw128_kmajor_desc(k_addr + (kk >> 2) * C::R_ATOM + (kk & 3) * 32),
                     sw128_kmajor_desc(qb + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        if (DK) {
          if (!mbar_wait(y_full, (uint32_t)t & 1u, status, P5_ERR_WAIT_ATTN)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C::HD / 16; ++kk)
            tc_mma_f16(sb + C::DP_COL, sw128_kmajor_desc(v_addr + (kk >> 2) * C::R_ATOM + (kk & 3) * 32),
                       sw128_kmajor_desc(y_addr + (kk >> 2) * C::BOX + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(y_empty);
        tc_commit(&sd_full[bt]);
        return true;
      };
      bool ok = mbar_wait(r_full, 0, status, P5_ERR_WAIT_ATTN);
      tc_fence_after();
      if (ok && n > 0) ok = issue_s(0);
      for (int i = 0; i < n && ok; ++i) {
        if (i + 1 < n && !issue_s(i + 1)) {
          ok = false;
          break;
        }
        const int bt = i & 1;
        if (!mbar_wait(&e_full[bt], (uint32_t)(i >> 1) & 1u, status, P5_ERR_WAIT_ATTN) ||
            (!DK && !mbar_wait(&x_full[bt], (uint32_t)(i >> 1) & 1u, status, P5_ERR_WAIT_ATTN))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sb = tmem_base + (uint32_t)(bt * C::BUF_COLS), xb = x_addr + bt * C::SLOT;
        // P^T / dS^T of query columns [16kk, 16kk+16): warpgroup kk/2's 16 columns at 32 (kk/2)
#pragma unroll
        for (int kk = 0; kk < C::QT / 16; ++kk)
          tc_mma_f16_ta(tmem_base + C::ACC_COL, sb + (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8),
                        sw128_mnmajor_desc(xb + kk * 2048, C::BOX), idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&x_empty[bt]);
      }
      if (!ok) flags[0] = 1;
      tc_commit(o_full);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- P^T / dS^T: thread = key = TMEM lane, warpgroup g takes query columns [32g, 32g+32)
    const int g = (warp - 4) >> 2, sub = warp & 3;
    const int r = sub * 32 + lane, key = k0 + r;
    const uint32_t t_lane = tmem_base + ((uint32_t)(sub * 32) << 16);
    bool alive = true;
    for (int i = 0; i < n; ++i) {
      const int bt = i & 1;
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
      bool ok = !flags[0] && mbar_wait(&sd_full[bt], (uint32_t)(i >> 1) & 1u, status, P5_ERR_WAIT_ATTN);
      if (__any_sync(0xffffffffu, !ok)) {
        flags[0] = 1;
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = t_lane + (uint32_t)(bt * C::BUF_COLS + 32 * g);
      uint32_t rs[32], rp[32];
      tmem_ld32(sb, rs);
      if (DK) tmem_ld32(sb + C::DP_COL, rp);
      tmem_wait_ld();
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
      tmem_st16(sb, pk);  // over this warpgroup's own S^T columns, already read
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&e_full[bt]);
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

}  // namespace p5

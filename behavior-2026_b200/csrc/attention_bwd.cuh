// attention_bwd.cuh — backward of the MQA attention (8 query heads share one 256-wide KV head).
//
// Rows are the folded (token, head) pairs of the forward kernel.  With P = exp(S - LSE), S = q k^T
// (q already scaled by 1/16) and D[row] = sum_d dO*O:
//   dS = P * (dO V^T - D),  dQ = dS K,  dK = dS^T Q,  dV = P^T dO.
// Three kernels, each with one fp32 accumulator in registers (the 256-wide head does not leave room
// for two): dQ per 64-row query block looping over key tiles; dK and dV per 64-key tile looping over
// the query rows that attend it.  Prefix keys are attended by the prefix queries and by the action
// queries of the same sample, so their kernels walk two query segments in a fixed order.
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace p5 {

struct QSeg {  // query rows of one batch item b: T tokens x 8 heads
  const bf16* q;
  int ldq;
  long qb;
  const bf16* dO;
  int ldo;
  long ob;
  const float* lse;  // [b*lb + row]
  const float* Dv;
  long lb;
  int T;
};

struct AttnBwdArgs {
  // keys (two segments, as in the forward)
  const bf16* k1;
  const bf16* v1;
  int ld1, len1;
  long b1stride;
  const bf16* k2;
  const bf16* v2;
  int ld2, len2;
  long b2stride;
  // dQ kernel: the query segment and where dq goes ([b*qb + tok*ld + h*256])
  QSeg qs;
  bf16* dq;
  int ld_dq;
  long dq_b;
  // dK/dV kernels: the keys of segment `kseg` (1 or 2), the query segments that attend them
  int kseg;
  QSeg qa, qbseg;
  int nq;  // 1 or 2 query segments
  bf16* dk;
  bf16* dv;
  int ld_dkv;
  long dkv_b;
};

constexpr int ABW_LDS = 256 + 8;
constexpr int ABW_TILE = 64 * ABW_LDS;  // elements

__device__ __forceinline__ void abw_load_rows(bf16* dst, const bf16* base, long bstride, int b, int ld, int r0,
                                              int nrows_valid, int col_of_row_mode) {
  // col_of_row_mode: 0 = plain rows (keys: row r at base + r*ld), 1 = folded MQA rows (token r/8, head r%8)
  for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
    const int r = i / 32, ch = i % 32;
    const int row = r0 + r;
    const bool ok = row < nrows_valid;
    const bf16* src = base;
    if (ok) {
      src = col_of_row_mode ? base + b * bstride + (long)(row / 8) * ld + (row % 8) * 256 + ch * 8
                            : base + b * bstride + (long)row * ld + ch * 8;
    }
    cp_async16(dst + r * ABW_LDS + ch * 8, src, ok);
  }
}

__device__ __forceinline__ void abw_load_keys(const AttnBwdArgs& a, int b, int j0, bf16* sK, bf16* sV) {
  const int total = a.len1 + a.len2;
  for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
    const int r = i / 32, ch = i % 32;
    const int j = j0 + r;
    const bool ok = j < total;
    const bf16* ks = a.k1;
    const bf16* vs = a.v1;
    if (ok && j < a.len1) {
      ks = a.k1 + b * a.b1stride + (long)j * a.ld1 + ch * 8;
      vs = a.v1 + b * a.b1stride + (long)j * a.ld1 + ch * 8;
    } else if (ok) {
      ks = a.k2 + b * a.b2stride + (long)(j - a.len1) * a.ld2 + ch * 8;
      vs = a.v2 + b * a.b2stride + (long)(j - a.len1) * a.ld2 + ch * 8;
    }
    cp_async16(sK + r * ABW_LDS + ch * 8, ks, ok);
    cp_async16(sV + r * ABW_LDS + ch * 8, vs, ok);
  }
}

// S[16 x 64] = A(16 rows of tile TA at arow) . B(64 rows of TB)^T over d = 256
__device__ __forceinline__ void abw_qk(float (&s)[8][4], const bf16* TA, int arow, const bf16* TB, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 16; ++ks) {
    uint32_t af[4];
    ldsm_x4(smem_u32(TA + (arow + (lane & 15)) * ABW_LDS + ks * 16 + (lane >> 4) * 8), af[0], af[1], af[2], af[3]);
#pragma unroll
    for (int nt = 0; nt < 8; nt += 2) {
      const int mi = lane >> 3;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(TB + (nt * 8 + (mi >> 1) * 8 + (lane & 7)) * ABW_LDS + ks * 16 + (mi & 1) * 8), b0, b1, b2,
              b3);
      mma_bf16_16816(s[nt], af, b0, b1);
      mma_bf16_16816(s[nt + 1], af, b2, b3);
    }
  }
}

// acc[16 x 256] += P(16 x 64, as packed A fragments) . T(64 rows x 256), T read transposed
__device__ __forceinline__ void abw_pv(float (&acc)[32][4], const uint32_t (&pf)[4][4], const bf16* T, int lane) {
  const int mi = lane >> 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t afr[4] = {pf[j][0], pf[j][1], pf[j][2], pf[j][3]};
#pragma unroll
    for (int dt = 0; dt < 32; dt += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(T + (j * 16 + (mi & 1) * 8 + (lane & 7)) * ABW_LDS + (dt + (mi >> 1)) * 8), b0, b1, b2, b3);
      mma_bf16_16816(acc[dt], afr, b0, b1);
      mma_bf16_16816(acc[dt + 1], afr, b2, b3);
    }
  }
}

__device__ __forceinline__ void pack_p(uint32_t (&pf)[4][4], const float (&p)[8][4]) {
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf2(p[nt][0], p[nt][1]);
    pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf2(p[nt][2], p[nt][3]);
  }
}

// ---------------------------------------------------------------- dQ
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const AttnBwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sO = sQ + ABW_TILE;  // dO
  bf16* sK = sO + ABW_TILE;
  bf16* sV = sK + ABW_TILE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const QSeg& qs = a.qs;
  const int rows = qs.T * P5_NH;
  const int r0 = blockIdx.x * 64;
  const int g = lane >> 2, cq = lane & 3;
  abw_load_rows(sQ, qs.q, qs.qb, b, qs.ldq, r0, rows, 1);
  abw_load_rows(sO, qs.dO, qs.ob, b, qs.ldo, r0, rows, 1);
  cp_async_commit();
  float lse[2], dd[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = r0 + warp * 16 + g + 8 * h;
    lse[h] = row < rows ? qs.lse[b * qs.lb + row] : 1e30f;
    dd[h] = row < rows ? qs.Dv[b * qs.lb + row] : 0.f;
  }
  float acc[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int total = a.len1 + a.len2;
  const float LOG2E = 1.4426950408889634f;
  for (int j0 = 0; j0 < total; j0 += 64) {
    __syncthreads();
    abw_load_keys(a, b, j0, sK, sV);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float s[8][4], dp[8][4];
    abw_qk(s, sQ, warp * 16, sK, lane);
    abw_qk(dp, sO, warp * 16, sV, lane);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j0 + nt * 8 + 2 * cq + (e & 1);
        const int h = e >> 1;
        const float p = key < total ? exp2f((s[nt][e] - lse[h]) * LOG2E) : 0.f;
        s[nt][e] = p * (dp[nt][e] - dd[h]);  // dS
      }
    uint32_t pf[4][4];
    pack_p(pf, s);
    abw_pv(acc, pf, sK, lane);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = r0 + warp * 16 + g + 8 * h;
    if (row >= rows) continue;
    bf16* dst = a.dq + b * a.dq_b + (long)(row / 8) * a.ld_dq + (row % 8) * 256;
#pragma unroll
    for (int dt = 0; dt < 32; ++dt)
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * cq) = pack_bf2(acc[dt][2 * h], acc[dt][2 * h + 1]);
  }
}

// ---------------------------------------------------------------- dK / dV (one kernel, `want_dk` picks the output)
template <bool DK>
__global__ void __launch_bounds__(128) attn_bwd_dkv_kernel(const AttnBwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sK = reinterpret_cast<bf16*>(smem_raw);
  bf16* sV = sK + ABW_TILE;
  bf16* sQ = sV + ABW_TILE;
  bf16* sO = sQ + ABW_TILE;  // dO
  float* sL = reinterpret_cast<float*>(sO + ABW_TILE);  // lse[64], D[64]
  float* sD = sL + 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int g = lane >> 2, cq = lane & 3;
  // this CTA's 64 keys: segment kseg, keys [k0, k0+64)
  const int seg_len = a.kseg == 1 ? a.len1 : a.len2;
  const int k0 = blockIdx.x * 64;
  {
    const bf16* kb = a.kseg == 1 ? a.k1 : a.k2;
    const bf16* vb = a.kseg == 1 ? a.v1 : a.v2;
    const int ld = a.kseg == 1 ? a.ld1 : a.ld2;
    const long bs = a.kseg == 1 ? a.b1stride : a.b2stride;
    abw_load_rows(sK, kb, bs, b, ld, k0, seg_len, 0);
    abw_load_rows(sV, vb, bs, b, ld, k0, seg_len, 0);
  }
  cp_async_commit();
  float acc[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const float LOG2E = 1.4426950408889634f;
  for (int sg = 0; sg < a.nq; ++sg) {
    const QSeg& qs = sg == 0 ? a.qa : a.qbseg;
    const int rows = qs.T * P5_NH;
    for (int r0 = 0; r0 < rows; r0 += 64) {
      __syncthreads();
      abw_load_rows(sQ, qs.q, qs.qb, b, qs.ldq, r0, rows, 1);
      abw_load_rows(sO, qs.dO, qs.ob, b, qs.ldo, r0, rows, 1);
      for (int i = threadIdx.x; i < 64; i += blockDim.x) {
        const int row = r0 + i;
        sL[i] = row < rows ? qs.lse[b * qs.lb + row] : 1e30f;
        sD[i] = row < rows ? qs.Dv[b * qs.lb + row] : 0.f;
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
      // S^T (16 keys x 64 rows) = K Q^T
      float st[8][4];
      abw_qk(st, sK, warp * 16, sQ, lane);
      float dpt[8][4];
      if (DK) abw_qk(dpt, sV, warp * 16, sO, lane);  // dP^T = V dO^T
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = nt * 8 + 2 * cq + (e & 1);
          const float p = exp2f((st[nt][e] - sL[col]) * LOG2E);
          st[nt][e] = DK ? p * (dpt[nt][e] - sD[col]) : p;
        }
      uint32_t pf[4][4];
      pack_p(pf, st);
      abw_pv(acc, pf, DK ? sQ : sO, lane);
    }
  }
  bf16* out = DK ? a.dk : a.dv;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int key = k0 + warp * 16 + g + 8 * h;
    if (key >= seg_len) continue;
    bf16* dst = out + b * a.dkv_b + (long)key * a.ld_dkv;
#pragma unroll
    for (int dt = 0; dt < 32; ++dt)
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * cq) = pack_bf2(acc[dt][2 * h], acc[dt][2 * h + 1]);
  }
}

constexpr int ABW_SMEM_DQ = 4 * ABW_TILE * 2;
constexpr int ABW_SMEM_DKV = 4 * ABW_TILE * 2 + 128 * 4;

}  // namespace p5

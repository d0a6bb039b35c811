// attention.cuh — fused softmax attention over bf16 Q/K/V, fp32 logits and softmax.
//
// Layouts (all row-major, bf16):
//   MQA (Gemma prefix and action expert: 8 query heads share one 256-wide KV head):
//     the 8 heads of a token are folded into 8 consecutive "rows", so one K/V tile load serves all
//     heads.  Row r -> token r/8, head r%8; q/out column offset head*256; K/V column offset 0.
//   MHA (SigLIP: 16 heads of 72): rows are tokens; the head comes from blockIdx.y and offsets both
//     the q/out and the K/V columns by head*72.
// The key sequence of batch item b is the concatenation of two segments, so the action expert can
// attend to [cached prefix K/V (len1) || its own K/V (len2)] without copying.
// A CTA owns 64 rows (4 warps x 16) and walks the keys in tiles of 64 with an online softmax.  With
// `splits` > 1 the keys are divided among CTAs and the partial (O, m, l) are merged by
// attn_combine_kernel (split-KV for the 50-token action queries).
#pragma once
#include "common.cuh"

namespace p5 {

struct AttnArgs {
  const bf16* q;
  int ldq;
  long q_bstride;  // elements between batch items
  bf16* out;
  int ldo;
  long o_bstride;
  const bf16* k1;
  const bf16* v1;
  int ld1, len1;
  long b1stride;
  const bf16* k2;
  const bf16* v2;
  int ld2, len2;
  long b2stride;
  int T;            // query tokens per batch item
  int G;            // heads folded into rows (8 for MQA, 1 for MHA)
  float qdiv;       // != 1: q <- R(q / qdiv) before use (SigLIP's 1/sqrt(72) step)
  int splits;       // key splits per (row block, batch item)
  int keys_per_split;
  float* ws_o;      // [batch*splits][rows][HD] unnormalised partial outputs
  float* ws_ml;     // [batch*splits][rows][2]   running max, running sum
  int pdl;
  float* lse;       // optional (splits == 1): log-sum-exp per row, [b * lse_b + row]
  long lse_b;
  int force_splits; // > 0: the tensor-core path uses this many key splits instead of choosing
  const int* valid1; // optional (tensor-core path): batch item b attends to the first valid1[b] keys of segment 1
  int group1;        // > 0 (tensor-core path): query tokens t < group1 attend to segment-1 keys j < group1 only
  int ws_half;       // 1 (tensor-core path): ws_o holds fp16 partials already divided by their own l
};

template <int HD, int NW = 4>
struct AttnCfg {
  static constexpr int HDP = (HD + 15) / 16 * 16;  // padded to the MMA K step
  static constexpr int LDS = HDP + 8;              // smem row stride (elements): conflict-free ldmatrix
  static constexpr int ROWS = 16 * NW, KT = 64;    // query rows per CTA (16 per warp), keys per tile
  static constexpr int TILE_ELEMS = KT * LDS;      // one K or V tile
  static constexpr int SMEM = (ROWS * LDS + 4 * TILE_ELEMS) * 2;  // Q + 2 x (K, V)
  static constexpr int ND = HD / 8;                                // output n-tiles of 8
};

template <int HD>
__device__ __forceinline__ void attn_load_kv(const AttnArgs& a, int b, int j0, int head_col, bf16* sK, bf16* sV) {
  using C = AttnCfg<HD, 4>;
  constexpr int CH = HD * 2 / 16;  // 16-byte chunks per row
  const int total = a.len1 + a.len2;
  for (int i = threadIdx.x; i < C::KT * CH; i += blockDim.x) {
    const int r = i / CH, ch = i % CH;
    const int j = j0 + r;
    const bf16* ks;
    const bf16* vs;
    bool ok = j < total;
    if (j < a.len1) {
      ks = a.k1 + b * a.b1stride + (long)j * a.ld1 + head_col;
      vs = a.v1 + b * a.b1stride + (long)j * a.ld1 + head_col;
    } else if (ok) {
      ks = a.k2 + b * a.b2stride + (long)(j - a.len1) * a.ld2 + head_col;
      vs = a.v2 + b * a.b2stride + (long)(j - a.len1) * a.ld2 + head_col;
    } else {
      ks = a.k1;
      vs = a.v1;
    }
    cp_async16(sK + r * C::LDS + ch * 8, ok ? (const void*)(ks + ch * 8) : (const void*)a.k1, ok);
    cp_async16(sV + r * C::LDS + ch * 8, ok ? (const void*)(vs + ch * 8) : (const void*)a.v1, ok);
  }
}

template <int HD, int NW>
__global__ void __launch_bounds__(32 * NW) attn_kernel(const AttnArgs a) {
  using C = AttnCfg<HD, NW>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* kv0 = sQ + C::ROWS * C::LDS;
  bf16* sK[2] = {kv0, kv0 + C::TILE_ELEMS};
  bf16* sV[2] = {kv0 + 2 * C::TILE_ELEMS, kv0 + 3 * C::TILE_ELEMS};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_total = a.T * a.G;
  const int r0 = blockIdx.x * C::ROWS;
  const int mha_head = a.G == 1 ? blockIdx.y : 0;
  const int kv_col = mha_head * HD;
  const int b = blockIdx.z / a.splits, split = blockIdx.z % a.splits;
  const int total = a.len1 + a.len2;
  const int kbeg = split * a.keys_per_split;
  const int kend = min(total, kbeg + a.keys_per_split);
  const int ntiles = (kend - kbeg + C::KT - 1) / C::KT;

  if (a.pdl) pdl_wait();

  // ---- Q tile (zero padding for columns >= HD and rows >= rows_total)
  {
    constexpr int CH = HD * 2 / 16;
    for (int i = threadIdx.x; i < C::ROWS * CH; i += blockDim.x) {
      const int r = i / CH, ch = i % CH;
      const int row = r0 + r;
      const bool ok = row < rows_total;
      const int tok = a.G > 1 ? row / a.G : row;
      const int hq = a.G > 1 ? row % a.G : mha_head;
      const bf16* src = a.q + b * a.q_bstride + (long)tok * a.ldq + hq * HD + ch * 8;
      cp_async16(sQ + r * C::LDS + ch * 8, ok ? (const void*)src : (const void*)a.q, ok);
    }
    if (C::HDP > HD) {
      for (int r = threadIdx.x; r < C::ROWS; r += blockDim.x)
        for (int c = HD; c < C::HDP; ++c) sQ[r * C::LDS + c] = tobf(0.f);
      for (int r = threadIdx.x; r < 2 * C::KT; r += blockDim.x) {
        bf16* k = (r < C::KT) ? sK[0] + r * C::LDS : sK[1] + (r - C::KT) * C::LDS;
        for (int c = HD; c < C::HDP; ++c) k[c] = tobf(0.f);
      }
    }
  }
  if (ntiles > 0) attn_load_kv<HD>(a, b, kbeg, kv_col, sK[0], sV[0]);
  cp_async_commit();

  float o[C::ND][4];
#pragma unroll
  for (int i = 0; i < C::ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.f, 0.f};
  const float LOG2E = 1.4426950408889634f;

  for (int it = 0; it < ntiles; ++it) {
    const int cur = it & 1;
    if (it + 1 < ntiles) attn_load_kv<HD>(a, b, kbeg + (it + 1) * C::KT, kv_col, sK[cur ^ 1], sV[cur ^ 1]);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0 && a.qdiv != 1.0f) {
      for (int i = threadIdx.x; i < C::ROWS * HD; i += blockDim.x) {
        bf16* p = sQ + (i / HD) * C::LDS + i % HD;
        *p = tobf(bf(*p) / a.qdiv);
      }
      __syncthreads();
    }
    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const bf16* kt = sK[cur];
#pragma unroll
    for (int ks = 0; ks < C::HDP / 16; ++ks) {
      uint32_t af[4];
      ldsm_x4(smem_u32(sQ + (warp * 16 + (lane & 15)) * C::LDS + ks * 16 + (lane >> 4) * 8), af[0], af[1], af[2],
              af[3]);
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3;
        ldsm_x4(smem_u32(kt + (nt * 8 + (mi >> 1) * 8 + (lane & 7)) * C::LDS + ks * 16 + (mi & 1) * 8), b0, b1, b2,
                b3);
        mma_bf16_16816(s[nt], af, b0, b1);
        mma_bf16_16816(s[nt + 1], af, b2, b3);
      }
    }
    // ---- mask keys beyond the segment end, online softmax
    const int j0 = kbeg + it * C::KT;
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int key = j0 + nt * 8 + 2 * cq;
      if (key >= kend) s[nt][0] = s[nt][2] = -1e30f;
      if (key + 1 >= kend) s[nt][1] = s[nt][3] = -1e30f;
    }
    float mt[2] = {-1e30f, -1e30f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mt[0] = fmaxf(mt[0], fmaxf(s[nt][0], s[nt][1]));
      mt[1] = fmaxf(mt[1], fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 1));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 2));
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float mn = fmaxf(m_run[h], mt[h]);
      alpha[h] = exp2f((m_run[h] - mn) * LOG2E);
      m_run[h] = mn;
      l_run[h] *= alpha[h];
    }
    uint32_t pf[4][4];  // P as A fragments: 4 key-steps of 16
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f((s[nt][0] - m_run[0]) * LOG2E), p1 = exp2f((s[nt][1] - m_run[0]) * LOG2E);
      const float p2 = exp2f((s[nt][2] - m_run[1]) * LOG2E), p3 = exp2f((s[nt][3] - m_run[1]) * LOG2E);
      l_run[0] += p0 + p1;
      l_run[1] += p2 + p3;
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf2(p0, p1);
      pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf2(p2, p3);
    }
#pragma unroll
    for (int dt = 0; dt < C::ND; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }
    // ---- O += P V
    const bf16* vt = sV[cur];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // A fragment order: (rows g, keys 0-7), (rows g+8, keys 0-7), (rows g, keys 8-15), (rows g+8, keys 8-15)
      const uint32_t afr[4] = {pf[j][0], pf[j][1], pf[j][2], pf[j][3]};
      const int mi = lane >> 3;
#pragma unroll
      for (int dt = 0; dt + 1 < C::ND; dt += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(vt + (j * 16 + (mi & 1) * 8 + (lane & 7)) * C::LDS + (dt + (mi >> 1)) * 8), b0, b1, b2, b3);
        mma_bf16_16816(o[dt], afr, b0, b1);
        mma_bf16_16816(o[dt + 1], afr, b2, b3);
      }
      if (C::ND & 1) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_u32(vt + (j * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * C::LDS + (C::ND - 1) * 8), b0, b1);
        mma_bf16_16816(o[C::ND - 1], afr, b0, b1);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- finish: reduce l over the quad, write normalised bf16 (or the split partials)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  const int g = lane >> 2, cq = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = r0 + warp * 16 + g + h * 8;
    if (row >= rows_total) continue;
    const int tok = a.G > 1 ? row / a.G : row;
    const int hq = a.G > 1 ? row % a.G : mha_head;
    if (a.splits == 1) {
      const float inv = l_run[h] > 0.f ? 1.0f / l_run[h] : 0.f;
      if (a.lse && cq == 0) a.lse[b * a.lse_b + row] = m_run[h] + logf(l_run[h]);
      bf16* dst = a.out + b * a.o_bstride + (long)tok * a.ldo + hq * HD;
#pragma unroll
      for (int dt = 0; dt < C::ND; ++dt)
        *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * cq) = pack_bf2(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
    } else {
      const long base = ((long)blockIdx.z * rows_total + row);
      float* dst = a.ws_o + base * HD;
#pragma unroll
      for (int dt = 0; dt < C::ND; ++dt)
        *reinterpret_cast<float2*>(dst + dt * 8 + 2 * cq) = make_float2(o[dt][2 * h], o[dt][2 * h + 1]);
      if (cq == 0) {
        a.ws_ml[base * 2] = m_run[h];
        a.ws_ml[base * 2 + 1] = l_run[h];
      }
    }
  }
  if (a.pdl) pdl_launch_dependents();
}

// merge split-KV partials: out = sum_s O_s e^(m_s - M) / sum_s l_s e^(m_s - M); item = (b, row, pair).
// With ws_half the partials are O_s / l_s in fp16, weighted by l_s e^(m_s - M) instead.
template <int HD>
__device__ __forceinline__ void attn_combine_item(const AttnArgs& a, long idx) {
  const int rows_total = a.T * a.G;
  const int d2 = idx % (HD / 2);
  const long br = idx / (HD / 2);
  const int row = br % rows_total, b = br / rows_total;
  float M = -1e30f, L = 0.f, o0 = 0.f, o1 = 0.f;
  constexpr int SMAX = 16;
  if (a.ws_half && a.splits <= SMAX) {
    const __half2* wh = reinterpret_cast<const __half2*>(a.ws_o);
    float2 ml[SMAX];
    __half2 ov[SMAX];
#pragma unroll
    for (int k = 0; k < SMAX; ++k) {
      const long base = ((long)b * a.splits + min(k, a.splits - 1)) * rows_total + row;
      ml[k] = *reinterpret_cast<const float2*>(a.ws_ml + base * 2);
      ov[k] = wh[base * (HD / 2) + d2];
    }
#pragma unroll
    for (int k = 0; k < SMAX; ++k) M = k < a.splits ? fmaxf(M, ml[k].x) : M;
#pragma unroll
    for (int k = 0; k < SMAX; ++k) {
      if (k >= a.splits) break;
      const float w = ml[k].y * __expf(ml[k].x - M);
      const float2 p = __half22float2(ov[k]);
      L += w;
      o0 += p.x * w;
      o1 += p.y * w;
    }
  } else if (a.ws_half) {
    const __half2* wh = reinterpret_cast<const __half2*>(a.ws_o);
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.ws_ml[(((long)b * a.splits + s) * rows_total + row) * 2]);
    for (int s = 0; s < a.splits; ++s) {
      const long base = ((long)b * a.splits + s) * rows_total + row;
      const float w = a.ws_ml[base * 2 + 1] * __expf(a.ws_ml[base * 2] - M);
      const float2 p = __half22float2(wh[base * (HD / 2) + d2]);
      L += w;
      o0 += p.x * w;
      o1 += p.y * w;
    }
  } else if (a.splits <= SMAX) {
    // every split's loads in flight together: indices past the split count re-read the last split
    // (weight 0), so the loads carry no conditions; the sums still run in split order
    float2 ml[SMAX], ov[SMAX];
#pragma unroll
    for (int k = 0; k < SMAX; ++k) {
      const long base = ((long)b * a.splits + min(k, a.splits - 1)) * rows_total + row;
      ml[k] = *reinterpret_cast<const float2*>(a.ws_ml + base * 2);
      ov[k] = *reinterpret_cast<const float2*>(a.ws_o + base * HD + 2 * d2);
    }
#pragma unroll
    for (int k = 0; k < SMAX; ++k) M = k < a.splits ? fmaxf(M, ml[k].x) : M;
#pragma unroll
    for (int k = 0; k < SMAX; ++k) {
      if (k >= a.splits) break;
      const float w = __expf(ml[k].x - M);
      L += ml[k].y * w;
      o0 += ov[k].x * w;
      o1 += ov[k].y * w;
    }
  } else {
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.ws_ml[(((long)b * a.splits + s) * rows_total + row) * 2]);
    for (int s = 0; s < a.splits; ++s) {
      const long base = ((long)b * a.splits + s) * rows_total + row;
      const float w = __expf(a.ws_ml[base * 2] - M);
      L += a.ws_ml[base * 2 + 1] * w;
      const float2 p = *reinterpret_cast<const float2*>(a.ws_o + base * HD + 2 * d2);
      o0 += p.x * w;
      o1 += p.y * w;
    }
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const int tok = a.G > 1 ? row / a.G : row;
  const int hq = a.G > 1 ? row % a.G : 0;
  bf16* dst = a.out + b * a.o_bstride + (long)tok * a.ldo + hq * HD + 2 * d2;
  *reinterpret_cast<uint32_t*>(dst) = pack_bf2(o0 * inv, o1 * inv);
}

template <int HD>
__global__ void attn_combine_kernel(const AttnArgs a, int batch) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (a.pdl) pdl_wait();
  if (idx < (long)batch * a.T * a.G * (HD / 2)) attn_combine_item<HD>(a, idx);
  if (a.pdl) pdl_launch_dependents();
}

}  // namespace p5

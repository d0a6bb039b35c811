// kernels.cuh — the small kernels around the GEMMs and attention: weight fill from the seeded
// generator, image patchify, norms, RoPE + KV-cache write, text embedding gather, the fp32 action
// projections, the time MLP and the Euler update.  All are memory-bound; each reads its inputs once.
#pragma once
#include "common.cuh"

namespace p5 {

// ---------------------------------------------------------------- parameters
// dst[(row_off + r*row_step) * ld + c] = bf16(base + N(0,1)*scale) for logical element r*C + c
__global__ void fill_param_kernel(bf16* dst, long R, int Cc, int ld, long row_off, int row_step, uint64_t key,
                                  float scale, float base) {
  const long n = R * Cc;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / Cc;
    const int c = (int)(i % Cc);
    const uint16_t h = p5_param_bf(key, (uint64_t)i, scale, base);
    dst[(row_off + r * row_step) * ld + c] = __ushort_as_bfloat16(h);
  }
}

// normal draws rounded to bf16 (synthetic KV cache) or kept in fp32 (noise)
__global__ void fill_normal_bf16_kernel(bf16* dst, long n, uint64_t key, float scale, long idx_off) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = __ushort_as_bfloat16(p5_f2bf(p5_normal(key, (uint64_t)(idx_off + i), scale)));
}

// ---------------------------------------------------------------- SigLIP patchify
// images [n_img][224][224][3] u8 -> A [n_img*256][640] bf16 holding (2p - 255), zero for k >= 588.
// (2p-255) is an odd integer in [-255, 255], exact in bf16; the stem GEMM scales by 1/255 so the
// product equals the fp32 convolution of x = p/127.5 - 1.
__global__ void patchify_kernel(const uint8_t* img, bf16* A, int n_img) {
  const long total = (long)n_img * 256 * P5_SIG_KPAD;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int k = (int)(i % P5_SIG_KPAD);
    const long tok = i / P5_SIG_KPAD;
    float v = 0.f;
    if (k < P5_SIG_K) {
      const int im = (int)(tok / 256), pt = (int)(tok % 256);
      const int py = pt / 16, px = pt % 16;
      const int ky = k / 42, rem = k % 42, kx = rem / 3, ch = rem % 3;
      const uint8_t p = img[(((long)im * P5_IMG + py * 14 + ky) * P5_IMG + px * 14 + kx) * 3 + ch];
      v = 2.0f * (float)p - 255.0f;
    }
    A[i] = tobf(v);
  }
}

// ---------------------------------------------------------------- norms (one warp per row)
// flax LayerNorm, eps 1e-6, two-pass statistics in fp32
// The row is read once with 16-byte loads and kept in registers for both passes (D <= 8 * 256).
__global__ void layernorm_kernel(const bf16* x, bf16* y, const bf16* s, const bf16* b, int T, int D) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  if (warp >= T) return;
  const bf16* xr = x + (long)warp * D;
  constexpr int MAXC = 8;  // 16-byte chunks per lane
  float v[MAXC][8];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int i = (lane + 32 * c) * 8;
    if (i < D) {
      unpack8(*reinterpret_cast<const uint4*>(xr + i), v[c]);
#pragma unroll
      for (int q = 0; q < 8; ++q) sum += v[c][q];
    }
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)D;
  float var = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int i = (lane + 32 * c) * 8;
    if (i < D) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float d = v[c][q] - mean;
        var += d * d;
      }
    }
  }
  for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float inv = 1.0f / sqrtf(var / (float)D + 1e-6f);
  bf16* yr = y + (long)warp * D;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int i = (lane + 32 * c) * 8;
    if (i < D) {
      float sc[8], bb[8];
      unpack8(*reinterpret_cast<const uint4*>(s + i), sc);
      unpack8(*reinterpret_cast<const uint4*>(b + i), bb);
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[q] = pack_bf2((v[c][2 * q] - mean) * inv * sc[2 * q] + bb[2 * q],
                        (v[c][2 * q + 1] - mean) * inv * sc[2 * q + 1] + bb[2 * q + 1]);
      *reinterpret_cast<uint4*>(yr + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  pdl_launch_dependents();
}

// Gemma RMSNorm: y = R(x / sqrt(mean(x^2) + 1e-6) * R(1 + scale) [+ shift])
//   plain:    scale = per-feature parameter, shift = null, mod_ld = 0
//   adaptive: scale/shift rows of the modulation table, row (t / rows_per_mod) with stride mod_ld
__global__ void rmsnorm_kernel(const bf16* x, bf16* y, const bf16* scale, const bf16* shift, int T, int D,
                               int rows_per_mod, int mod_ld, int ld_y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  if (warp >= T) return;
  const bf16* xr = x + (long)warp * D;
  const long mrow = mod_ld ? (long)(warp / rows_per_mod) * mod_ld : 0;
  const bf16* sc = scale + mrow;
  const bf16* sh = shift ? shift + mrow : nullptr;
  float ss = 0.f;
  for (int i = lane * 8; i < D; i += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf2(w[q]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / (float)D + 1e-6f);
  bf16* yr = y + (long)warp * ld_y;
  for (int i = lane * 8; i < D; i += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 us = *reinterpret_cast<const uint4*>(sc + i);
    uint4 uh = make_uint4(0, 0, 0, 0);
    if (sh) uh = *reinterpret_cast<const uint4*>(sh + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w}, ws[4] = {us.x, us.y, us.z, us.w}, wh[4] = {uh.x, uh.y, uh.z, uh.w};
    uint32_t out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf2(w[q]), s2 = unpack_bf2(ws[q]), h2 = unpack_bf2(wh[q]);
      const float a = f.x * inv * rbf(1.0f + s2.x) + h2.x;
      const float c = f.y * inv * rbf(1.0f + s2.y) + h2.y;
      out[q] = pack_bf2(a, c);
    }
    *reinterpret_cast<uint4*>(yr + i) = make_uint4(out[0], out[1], out[2], out[3]);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- RoPE + KV write
// qkv [T][2560] (q: 8 heads x 256, k: 256, v: 256).  Token t has position pos_off + t % per_sample.
// q <- R(rope(q)) * 1/16 in place; kout[t] <- R(rope(k)); vout[t] <- v.
// RoPE pairs (i, i+128) of each 256-wide head (openpi gemma._apply_rope).
__global__ void rope_qkv_kernel(bf16* qkv, int T, int per_sample, int pos_off, bf16* kout, bf16* vout,
                                const float* cos_t, const float* sin_t, int ld_kv) {
  const int t = blockIdx.x;
  pdl_wait();
  if (t >= T) return;
  const int pos = pos_off + t % per_sample;
  const float* cs = cos_t + (long)pos * 128;
  const float* sn = sin_t + (long)pos * 128;
  bf16* row = qkv + (long)t * P5_QKV;
  // 9 rotated heads (8 q + 1 k) x 128 pairs + 256 v copies
  for (int i = threadIdx.x; i < 9 * 128 + 128; i += blockDim.x) {
    if (i < 9 * 128) {
      const int h = i / 128, j = i % 128;
      bf16* v = row + h * 256;
      const float x1 = bf(v[j]), x2 = bf(v[j + 128]);
      const float a = rbf(x1 * cs[j] - x2 * sn[j]);
      const float c = rbf(x2 * cs[j] + x1 * sn[j]);
      if (h < 8) {
        v[j] = tobf(a * 0.0625f);
        v[j + 128] = tobf(c * 0.0625f);
      } else {
        kout[(long)t * ld_kv + j] = tobf(a);
        kout[(long)t * ld_kv + j + 128] = tobf(c);
      }
    } else {
      const int j = (i - 9 * 128) * 2;
      *reinterpret_cast<uint32_t*>(vout + (long)t * ld_kv + j) =
          *reinterpret_cast<const uint32_t*>(row + 2304 + j);
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- text embedding
// x[b][768 + i] = R(table[tok] * 45.25)  for i < n_text (Gemma embedder scale sqrt(2048) in bf16)
__global__ void embed_text_kernel(const int32_t* tokens, const bf16* table, bf16* x, int n_text, int P,
                                  int img_tokens) {
  const int b = blockIdx.y, i = blockIdx.x;
  pdl_wait();
  long tok = tokens[(long)b * n_text + i];
  if (tok < 0 || tok >= P5_VOCAB) tok = 0;  // out-of-vocabulary ids read row 0 instead of out of bounds
  const bf16* src = table + tok * P5_GEM_W;
  bf16* dst = x + ((long)b * P + img_tokens + i) * P5_GEM_W;
  for (int d = threadIdx.x * 2; d < P5_GEM_W; d += blockDim.x * 2) {
    const float2 f = unpack_bf2(*reinterpret_cast<const uint32_t*>(src + d));
    *reinterpret_cast<uint32_t*>(dst + d) = pack_bf2(f.x * P5_EMBED_SCALE, f.y * P5_EMBED_SCALE);
  }
  pdl_launch_dependents();
}

// The text part of the prefix given as embeddings (pi05_prefill_embeds): rows [img_tokens, img_tokens +
// n_text) of each sample's prefix copied from the caller's bf16 rows; grid (n_text, n), 256 threads x 8.
__global__ void copy_text_emb_kernel(const bf16* emb, bf16* x, int n_text, int P, int img_tokens) {
  const int b = blockIdx.y, i = blockIdx.x;
  pdl_wait();
  const uint4* src = reinterpret_cast<const uint4*>(emb + ((long)b * n_text + i) * P5_GEM_W);
  uint4* dst = reinterpret_cast<uint4*>(x + ((long)b * P + img_tokens + i) * P5_GEM_W);
  for (int d = threadIdx.x; d < P5_GEM_W / 8; d += blockDim.x) dst[d] = src[d];
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- action projections (fp32 math)
// action_in_proj: y[t][o] = R(sum_k x[t][k] W[o][k] + b[o]), x fp32 [T][32] (nnx.Linear in fp32)
// ss_out (optional): per-token partial sums of squares of the stored outputs, one per 16 output
// features, ss_out[(o / 16) * ss_ld + t] (the fused adaRMSNorm of the next projection reads them);
// requires D % 32 == 0 so that every warp is whole.
__global__ void action_in_kernel(const float* xt, const bf16* W, const bf16* b, bf16* y, int T, int D,
                                 float* ss_out, int ss_ld) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  if (idx >= (long)T * D) return;
  const int t = (int)(idx / D), o = (int)(idx % D);
  // vector loads of the thread's weight row (64 B) and its token's state row (128 B); the sum still
  // runs over k in order
  const float4* x = reinterpret_cast<const float4*>(xt + (long)t * P5_ACT_D);
  const uint4* w = reinterpret_cast<const uint4*>(W + (long)o * P5_ACT_D);
  float acc = 0.f;
#pragma unroll
  for (int q = 0; q < P5_ACT_D / 8; ++q) {
    float wf[8];
    unpack8(w[q], wf);
    const float4 x0 = x[2 * q], x1 = x[2 * q + 1];
    acc += x0.x * wf[0];
    acc += x0.y * wf[1];
    acc += x0.z * wf[2];
    acc += x0.w * wf[3];
    acc += x1.x * wf[4];
    acc += x1.y * wf[5];
    acc += x1.z * wf[6];
    acc += x1.w * wf[7];
  }
  const bf16 yb = tobf(acc + bf(b[o]));
  y[idx] = yb;
  if (ss_out) {
    float sq = bf(yb) * bf(yb);
#pragma unroll
    for (int o2 = 8; o2; o2 >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o2);
    if ((threadIdx.x & 15) == 0) ss_out[(size_t)(o >> 4) * ss_ld + t] = sq;
  }
  pdl_launch_dependents();
}

// action_out_proj + Euler step, one warp per (token, action dim):
//   v = R(h[t] . W[j] + b[j]);  x[t][j] += R(dt_bf16 * v)
__global__ void action_out_euler_kernel(const bf16* h, const bf16* W, const bf16* b, float* xt, float* v_out, int T,
                                        int D, float dtb) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  if (w >= T * P5_ACT_D) return;
  const int t = w / P5_ACT_D, j = w % P5_ACT_D;
  const bf16* hr = h + (long)t * D;
  const bf16* wr = W + (long)j * D;
  float acc = 0.f;
  for (int k = lane * 8; k < D; k += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(hr + k), c = *reinterpret_cast<const uint4*>(wr + k);
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, cc[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf2(aa[q]), g = unpack_bf2(cc[q]);
      acc += f.x * g.x + f.y * g.y;
    }
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const float v = rbf(acc + bf(b[j]));
    if (v_out) v_out[(long)t * P5_ACT_D + j] = v;
    xt[(long)t * P5_ACT_D + j] += rbf(dtb * v);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- prompt padding
// valid[b] = image tokens + the prompt up to its last non-padding id (openpi pads prompts with id 0 and
// masks the padding); a prompt of padding only keeps its first token
__global__ void text_valid_kernel(const int32_t* tokens, int n, int n_text, int n_img_tokens, int* valid) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  const int32_t* t = tokens + (size_t)b * n_text;
  int len = n_text;
  while (len > 1 && t[len - 1] == 0) --len;
  valid[b] = n_img_tokens + len;
}

// ---------------------------------------------------------------- correlated noise
// z[k][i] = fp32(sum_{j <= i} L[i][j] eps[k][j]) with a lower-triangular L [dim][dim]: one warp per output, the
// lanes stride over j and accumulate in fp64 (a fixed-order reduction: reruns are bit-identical, and the fp64
// sum rounds to the same fp32 as any other fp64 order except at rare ties)
__global__ void correlate_noise_kernel(const float* L, const float* eps, float* z, int m, int dim) {
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long)m * dim) return;
  const int k = (int)(w / dim), i = (int)(w % dim);
  const float* Li = L + (size_t)i * dim;
  const float* ek = eps + (size_t)k * dim;
  double acc = 0.0;
  for (int j = lane; j <= i; j += 32) acc += (double)Li[j] * (double)ek[j];
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) z[(size_t)k * dim + i] = (float)acc;
}

// ---------------------------------------------------------------- soft inpainting (one CTA per sample)
// After an Euler step that lands at time t, for the samples whose known rows are on: the first K values
// of the chunk (K = fixed rows x 32) are put back on the flow path of the known actions,
// x_K <- t eps_K + (1 - t) a_K (eps the step-0 noise), and the rest follows the Gaussian conditional,
// x_U += C (x_K,new - x_K,old), C = Sigma_UO Sigma_OO^-1 [U][K].  Unfused fp32 for the known rows, the
// correction accumulated in fp64 (one warp per row of C) and rounded once.  Dynamic smem: K floats.
__global__ void inpaint_kernel(float* xt, const float* eps, const float* known, const int* on, const float* C,
                               int s0, int horizon, int K, float t) {
  extern __shared__ float delta[];
  const int b = blockIdx.x, sample = s0 + b;
  if (!on[sample]) return;  // uniform for the CTA
  const int n = horizon * P5_ACT_D, U = n - K;
  float* x = xt + (size_t)b * n;
  const float* e = eps + (size_t)b * n;
  const float* a = known + (size_t)sample * K;
  const float omt = __fsub_rn(1.0f, t);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = __fadd_rn(__fmul_rn(t, e[k]), __fmul_rn(omt, a[k]));
    delta[k] = __fsub_rn(v, x[k]);
    x[k] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int u = warp; u < U; u += nw) {
    const float* cr = C + (size_t)u * K;
    double acc = 0.0;
    for (int k = lane; k < K; k += 32) acc += (double)cr[k] * (double)delta[k];
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) x[K + u] = __fadd_rn(x[K + u], (float)acc);
  }
}

// ---------------------------------------------------------------- KV layer mixing (PiBehavior)
// dst_l = bf16(bf16(sum_j w[l][j] src_j) + bias[l]) over the prefix cache's L layers, for the samples
// [s0, s0 + n): one thread per 8 head dims of one (sample, position), holding that slice of every layer
// in registers, so each cache element is read once and each mixed element written once.  w [L][L] and
// bias [L][256] hold bf16 values; the sum runs over j in order in fp32 without contraction.
constexpr int P5_KV_MIX_MAX_LAYERS = 18;
__global__ void kv_mix_kernel(const bf16* src, bf16* dst, const float* w, const float* bias, int L, long layer_stride,
                              long first, long items) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= items) return;
  const long off = first + i * 8;  // element offset inside a layer
  const int d0 = (int)(off % P5_HD);
  uint4 x[P5_KV_MIX_MAX_LAYERS];
#pragma unroll
  for (int j = 0; j < P5_KV_MIX_MAX_LAYERS; ++j)
    if (j < L) x[j] = *reinterpret_cast<const uint4*>(src + j * layer_stride + off);
  for (int l = 0; l < L; ++l) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < P5_KV_MIX_MAX_LAYERS; ++j) {
      if (j < L) {
        const float wj = w[l * L + j];
        float f[8];
        unpack8(x[j], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(wj, f[q]));
      }
    }
    const float* b = bias + (long)l * P5_HD + d0;
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = pack_bf2(rbf(acc[2 * q]) + b[2 * q], rbf(acc[2 * q + 1]) + b[2 * q + 1]);
    *reinterpret_cast<uint4*>(dst + l * layer_stride + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------- time MLP (fp32, one warp per output)
// y[s][o] = swish(sum_k x[s][k] W[o][k] + b[o]); optional bf16 copy (input of the bf16 modulation Dense)
__global__ void linear_swish_f32_kernel(const float* x, const bf16* W, const bf16* b, float* y, bf16* ybf, int S,
                                        int D) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= S * D) return;
  const int s = w / D, o = w % D;
  const float* xr = x + (long)s * D;
  const bf16* wr = W + (long)o * D;
  float acc = 0.f;
  for (int k = lane; k < D; k += 32) acc += xr[k] * bf(wr[k]);
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const float v = acc + bf(b[o]);
    const float sw = v / (1.0f + expf(-v));
    y[(long)s * D + o] = sw;
    if (ybf) ybf[(long)s * D + o] = tobf(sw);
  }
}

}  // namespace p5

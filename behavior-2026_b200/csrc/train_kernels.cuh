// train_kernels.cuh — kernels of the LoRA train step (backward pass, loss, optimizer).
//
// The step follows the openpi training loss the reference engine ported (π05_네이티브엔진.md:206-229,
// openpi models/pi0.py:189-214): x_t = t*noise + (1-t)*actions, u = noise - actions, v = net(x_t, t, prefix),
// loss = mean((v-u)^2); trainable parameters are rank-16 LoRA adapters on q/k/v/o/gate/up/down of the
// Gemma-2B prefix and the action expert; everything else is frozen.  Gradients flow in fp32 where they
// are reduced and in bf16 where they feed a tensor-core GEMM.
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace p5 {

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  return gelu_tanh_grad_s(x, half_one_plus_tanh(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

// ---------------------------------------------------------------- loss
// x_t = t*eps + (1-t)*a ; u = eps - a   (per sample t), fp32
__global__ void flow_inputs_kernel(const float* eps, const float* act, const float* t, float* xt, float* u, int H,
                                   int n) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)n * H * P5_ACT_D) return;
  const int b = (int)(i / ((long)H * P5_ACT_D));
  const float tb = t[b];
  xt[i] = tb * eps[i] + (1.0f - tb) * act[i];
  u[i] = eps[i] - act[i];
}

// v = R(h . Wout^T + b) (bf16 Linear), per-row squared error sum, dv = 2 (v - u) / count
__global__ void out_proj_loss_kernel(const bf16* h, const bf16* W, const bf16* b, const float* u, float* dv,
                                     float* row_loss, int T, int D, float inv_count) {
  const int t = blockIdx.x;
  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;  // 32 warps = 32 action dims
  if (t >= T) return;
  const bf16* hr = h + (long)t * D;
  const bf16* wr = W + (long)j * D;
  float acc = 0.f;
  for (int k = lane * 8; k < D; k += 256) {
    float a8[8], w8[8];
    const uint4 ua = *reinterpret_cast<const uint4*>(hr + k), uw = *reinterpret_cast<const uint4*>(wr + k);
    const uint32_t aa[4] = {ua.x, ua.y, ua.z, ua.w}, ww[4] = {uw.x, uw.y, uw.z, uw.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf2(aa[q]), g = unpack_bf2(ww[q]);
      a8[2 * q] = f.x; a8[2 * q + 1] = f.y; w8[2 * q] = g.x; w8[2 * q + 1] = g.y;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) acc += a8[q] * w8[q];
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float sq[32];
  if (lane == 0) {
    const float v = rbf(acc + bf(b[j]));
    const float e = v - u[(long)t * P5_ACT_D + j];
    dv[(long)t * P5_ACT_D + j] = 2.0f * e * inv_count;
    sq[j] = e * e;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < 32; ++i) s += sq[i];
    row_loss[t] = s;
  }
}

// deterministic sum of per-row losses (one block)
__global__ void sum_rows_kernel(const float* rows, int n, float scale, float* out) {
  __shared__ float part[256];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) s += rows[i];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out += part[0] * scale;
}

// dh[t][k] = sum_j dv[t][j] Wout[j][k]  (action_out_proj backward, frozen weight)
__global__ void out_proj_bwd_kernel(const float* dv, const bf16* W, bf16* dh, int T, int D) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * D) return;
  const int t = (int)(i / D), k = (int)(i % D);
  float acc = 0.f;
#pragma unroll 8
  for (int j = 0; j < P5_ACT_D; ++j) acc += dv[(long)t * P5_ACT_D + j] * bf(W[(long)j * D + k]);
  dh[i] = tobf(acc);
}

// ---------------------------------------------------------------- norm backward (one warp per row)
// y = n*w + shift with n = x*rstd, w = R(1+scale) (plain: scale per feature; adaptive: per-sample row
// of the modulation table).  dx (+)= rstd * (dn - n * mean(dn*n)), dn = dy*w.
__global__ void rmsnorm_bwd_kernel(const bf16* x, const bf16* dy, int ld_dy, const bf16* scale, int rows_per_mod,
                                   int mod_ld, float* dx_acc, int T, int D) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const bf16* xr = x + (long)warp * D;
  const bf16* dr = dy + (long)warp * ld_dy;
  const bf16* sc = scale + (mod_ld ? (long)(warp / rows_per_mod) * mod_ld : 0);
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float v = bf(xr[i]);
    ss += v * v;
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = 1.0f / sqrtf(ss / (float)D + 1e-6f);
  float dot = 0.f;
  for (int i = lane; i < D; i += 32) dot += bf(dr[i]) * rbf(1.0f + bf(sc[i])) * bf(xr[i]) * rstd;
  for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  const float m = dot / (float)D;
  float* out = dx_acc + (long)warp * D;
  for (int i = lane; i < D; i += 32) {
    const float n = bf(xr[i]) * rstd;
    const float dn = bf(dr[i]) * rbf(1.0f + bf(sc[i]));
    out[i] += rstd * (dn - n * m);
  }
}

// The same for D = 256 * CH: a warp keeps its row in registers (8 consecutive elements per lane and
// chunk, 16-byte loads; x is read once instead of three times) and updates dx_acc with 16-byte stores.
template <int CH>
__global__ void rmsnorm_bwd_vec_kernel(const bf16* x, const bf16* dy, int ld_dy, const bf16* scale, int rows_per_mod,
                                       int mod_ld, float* dx_acc, int T) {
  constexpr int D = 256 * CH;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const bf16* xr = x + (long)warp * D;
  const bf16* dr = dy + (long)warp * ld_dy;
  const bf16* sc = scale + (mod_ld ? (long)(warp / rows_per_mod) * mod_ld : 0);
  uint4 xv[CH], dv[CH], sv[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int i = (c * 32 + lane) * 8;
    xv[c] = *reinterpret_cast<const uint4*>(xr + i);
    dv[c] = *reinterpret_cast<const uint4*>(dr + i);
    sv[c] = *reinterpret_cast<const uint4*>(sc + i);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float xf[8];
    unpack8(xv[c], xf);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += xf[k] * xf[k];
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = 1.0f / sqrtf(ss / (float)D + 1e-6f);
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float xf[8], df[8], sf[8];
    unpack8(xv[c], xf);
    unpack8(dv[c], df);
    unpack8(sv[c], sf);
#pragma unroll
    for (int k = 0; k < 8; ++k) dot += df[k] * rbf(1.0f + sf[k]) * xf[k] * rstd;
  }
  for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  const float m = dot / (float)D;
  float* out = dx_acc + (long)warp * D;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int i = (c * 32 + lane) * 8;
    float xf[8], df[8], sf[8];
    unpack8(xv[c], xf);
    unpack8(dv[c], df);
    unpack8(sv[c], sf);
    float4* o4 = reinterpret_cast<float4*>(out + i);
    float4 a0 = o4[0], a1 = o4[1];
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = rstd * (df[k] * rbf(1.0f + sf[k]) - xf[k] * rstd * m);
    a0.x += r[0];
    a0.y += r[1];
    a0.z += r[2];
    a0.w += r[3];
    a1.x += r[4];
    a1.y += r[5];
    a1.z += r[6];
    a1.w += r[7];
    o4[0] = a0;
    o4[1] = a1;
  }
}

// fp32 residual-stream gradient -> bf16, 8 elements per thread (D % 8 == 0), optionally times the
// per-sample gate (gated residual backward)
__global__ void grad_to_bf16_vec_kernel(const float* g, bf16* out, int ld_out, const bf16* gate, int rows_per_gate,
                                        int gate_ld, int T, int D) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int dc = D / 8;
  if (i >= (long)T * dc) return;
  const int t = (int)(i / dc), k = (int)(i % dc) * 8;
  const float4* src = reinterpret_cast<const float4*>(g + (long)t * D + k);
  const float4 u = src[0], w = src[1];
  float v[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
  if (gate) {
    float gf[8];
    unpack8(*reinterpret_cast<const uint4*>(gate + (long)(t / rows_per_gate) * gate_ld + k), gf);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] *= gf[q];
  }
  *reinterpret_cast<uint4*>(out + (long)t * ld_out + k) =
      make_uint4(pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]), pack_bf2(v[4], v[5]), pack_bf2(v[6], v[7]));
}

// fp32 residual-stream gradient -> bf16 (optionally times the per-sample gate: gated residual backward)
__global__ void grad_to_bf16_kernel(const float* g, bf16* out, int ld_out, const bf16* gate, int rows_per_gate,
                                    int gate_ld, int T, int D) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * D) return;
  const int t = (int)(i / D), k = (int)(i % D);
  float v = g[i];
  if (gate) v *= bf(gate[(long)(t / rows_per_gate) * gate_ld + k]);
  out[(long)t * ld_out + k] = tobf(v);
}

// GeGLU backward: gu interleaved [T][2F] (gate 2j, up 2j+1), dact [T][F] (ld) -> dgu [T][2F] (ld)
// 8 consecutive (gate, up) pairs per thread (F % 8 == 0): 32-byte gate/up loads, 16-byte dact loads and
// stores, one tanh per pair for both the GELU value and its derivative.
__global__ void geglu_bwd_kernel(const bf16* gu, const bf16* dact, int ld_dact, bf16* dgu, int ld_dgu, int T,
                                 int F) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int fc = F / 8;
  if (i >= (long)T * fc) return;
  const int t = (int)(i / fc), j0 = (int)(i % fc) * 8;
  const uint4* g4 = reinterpret_cast<const uint4*>(gu + (long)t * 2 * F + 2 * j0);
  const uint4 ga = g4[0], gb = g4[1];
  const uint4 dv = *reinterpret_cast<const uint4*>(dact + (long)t * ld_dact + j0);
  const uint32_t gw[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
  float da[8];
  unpack8(dv, da);
  uint32_t o[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float2 p = unpack_bf2(gw[k]);
    o[k] = geglu_bwd_pair(p.x, p.y, da[k]);
  }
  uint4* dst = reinterpret_cast<uint4*>(dgu + (long)t * ld_dgu + 2 * j0);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// RoPE backward on the attention gradients in dqkv (ld): q part was R(rope(q))*1/16, k part R(rope(k)).
// The inverse rotation of the pair (i, i+128) by angle a is rotation by -a.
__global__ void rope_bwd_kernel(bf16* dqkv, int ld, int T, int per_sample, int pos_off, const float* cos_t,
                                const float* sin_t, int do_q) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const int pos = pos_off + t % per_sample;
  const float* cs = cos_t + (long)pos * 128;
  const float* sn = sin_t + (long)pos * 128;
  bf16* row = dqkv + (long)t * ld;
  for (int i = threadIdx.x; i < 9 * 128; i += blockDim.x) {
    const int h = i / 128, j = i % 128;
    if (h < 8 && !do_q) continue;
    bf16* v = row + h * 256;
    const float sc = h < 8 ? 0.0625f : 1.0f;
    const float a = bf(v[j]) * sc, c = bf(v[j + 128]) * sc;
    v[j] = tobf(a * cs[j] + c * sn[j]);
    v[j + 128] = tobf(c * cs[j] - a * sn[j]);
  }
}

// D[row] = sum_d dO[row][d] * O[row][d] for the folded MQA rows (token t, head h)
__global__ void attn_dot_kernel(const bf16* dO, int ld_do, const bf16* O, int ld_o, float* D, int T) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * P5_NH) return;
  const int t = warp / P5_NH, h = warp % P5_NH;
  const bf16* a = dO + (long)t * ld_do + h * P5_HD;
  const bf16* b = O + (long)t * ld_o + h * P5_HD;
  float s = 0.f;
  for (int d = lane; d < P5_HD; d += 32) s += bf(a[d]) * bf(b[d]);
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) D[warp] = s;
}

// ---------------------------------------------------------------- LoRA parameter plumbing
// Scatter fp32 adapters into the bf16 operands of the GEMMs (after init and every optimizer step).
struct LoraScatter {
  const float* A;  // [16][K]
  const float* B;  // [Fa][16]
  int K, Fa;
  // forward weight: Wf[row(f)][colB + j] = B[f][j]; backward weight Wb[k][colA + j] = A[j][k]
  bf16* Wf;
  int ld_wf, colB, row_off, row_step;
  bf16* Wb;
  int ld_wb, colA;
  bf16* Acat;  // rows [16a, 16a+16) = A : [16n][K]
  bf16* Btcat;  // Btcat[16a + j][row(f)] = B[f][j] : [16n][F]
  int ld_bt, arow;
};
__global__ void lora_scatter_kernel(LoraScatter s) {
  const long nA = 16L * s.K, nB = (long)s.Fa * 16;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nA + nB; i += (long)gridDim.x * blockDim.x) {
    if (i < nA) {
      const int j = (int)(i / s.K), k = (int)(i % s.K);
      const bf16 v = tobf(s.A[i]);
      s.Wb[(long)k * s.ld_wb + s.colA + j] = v;
      s.Acat[(long)(s.arow + j) * s.K + k] = v;
    } else {
      const long q = i - nA;
      const int f = (int)(q / 16), j = (int)(q % 16);
      const bf16 v = tobf(s.B[q]);
      const long row = (long)s.row_off + (long)f * s.row_step;
      s.Wf[row * s.ld_wf + s.colB + j] = v;
      s.Btcat[(long)(s.arow + j) * s.ld_bt + row] = v;
    }
  }
}

// copy a frozen [F][K] weight into the forward [F][K+extra] and the transposed backward [K][F+extra] buffers
__global__ void lora_frozen_copy_kernel(const bf16* W, int F, int K, bf16* Wf, int ld_wf, bf16* Wb, int ld_wb) {
  const long n = (long)F * K;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int f = (int)(i / K), k = (int)(i % K);
    const bf16 v = W[i];
    Wf[(long)f * ld_wf + k] = v;
    Wb[(long)k * ld_wb + f] = v;
  }
}

// x[i] *= s: re-weights a running mean when more samples join it
__global__ void scale_f32_kernel(float* x, long n, float s) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) x[i] *= s;
}

// ema = d * ema + (1 - d) * p after each update (openpi scripts/train.py)
__global__ void ema_kernel(float* ema, const float* p, long n, float d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    ema[i] = d * ema[i] + (1.0f - d) * p[i];
}

// ---------------------------------------------------------------- optimizer
// sum of squares of the gradient, deterministic two-level reduction
__global__ void sumsq_partial_kernel(const float* g, long n, float* partial) {
  __shared__ float part[256];
  float s = 0.f;
  for (long i = (long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long)gridDim.x * 256) s += g[i] * g[i];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = part[0];
}

// AdamW (optax order: clip_by_global_norm -> adam moments -> bias correction -> + wd * p -> * -lr)
__global__ void adamw_kernel(float* p, const float* g, float* m, float* v, long n, const float* sumsq_partial,
                             int n_partial, float clip, float lr, float b1, float b2, float eps, float wd, int step) {
  __shared__ float scale_s;
  if (threadIdx.x == 0) {
    float ss = 0.f;
    for (int i = 0; i < n_partial; ++i) ss += sumsq_partial[i];
    const float norm = sqrtf(ss);
    scale_s = (clip > 0.f && norm > clip) ? clip / norm : 1.0f;
  }
  __syncthreads();
  const float sc = scale_s;
  const float c1 = 1.0f - powf(b1, (float)step), c2 = 1.0f - powf(b2, (float)step);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gi = g[i] * sc;
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float upd = (mi / c1) / (sqrtf(vi / c2) + eps) + wd * p[i];
    p[i] -= lr * upd;
  }
}

__global__ void lora_init_kernel(float* p, long n, uint64_t seed, float scale) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    p[i] = p5_bf2f(p5_f2bf(p5_normal(seed, (uint64_t)i, scale)));
}

}  // namespace p5

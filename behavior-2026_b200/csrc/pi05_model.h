/*
 * pi05_model.h — shapes of the pi0.5 network and the seeded synthetic generator.
 *
 * Shapes follow the engine record of the reference (docs/archive/windows/π05_네이티브엔진.md:28-31):
 *   SigLIP So400m/14: width 1152, 27 layers, MLP 4304, 16 heads x 72, 224^2 -> 256 tokens per camera
 *   Gemma-2B prefix:  width 2048, 18 layers, MLP 16384, 8 query heads, 1 KV head, head dim 256
 *   Gemma-300M expert: width 1024, 18 layers, MLP 4096, same attention geometry, adaRMSNorm on time
 *
 * The generator is counter based: every scalar of every tensor is a pure function of
 * (seed, tensor kind, layer or sample, logical flat index).  The same code runs on the host
 * (CPU oracle, host-side input generation) and on the device (weight fill kernel), and it uses
 * only integer arithmetic plus one IEEE multiply (and one add for offset tensors), so both sides
 * produce the same bits.  Normals are Irwin-Hall sums of eight 16-bit uniforms scaled to unit
 * variance (bounded at +-4.9 sigma), which stands in for N(0, s^2).
 *
 * Host code that includes this header must be compiled with -ffp-contract=off.
 */
#ifndef PI05_MODEL_H
#define PI05_MODEL_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define P5_FN __host__ __device__ __forceinline__
#else
#define P5_FN static inline
#endif

/* ---- fixed widths (depths are run-time configuration) ---- */
enum {
  P5_SIG_W = 1152, P5_SIG_MLP = 4304, P5_SIG_HEADS = 16, P5_SIG_HD = 72,
  P5_SIG_PATCH = 14, P5_IMG = 224, P5_SIG_TOK = 256, P5_SIG_K = 588, P5_SIG_KPAD = 640,
  P5_SIG_QKV = 3 * 1152,
  P5_GEM_W = 2048, P5_GEM_MLP = 16384, P5_VOCAB = 257152,
  P5_EXP_W = 1024, P5_EXP_MLP = 4096,
  P5_NH = 8, P5_HD = 256, P5_QDIM = 8 * 256, P5_QKV = 8 * 256 + 2 * 256,
  P5_ACT_D = 32,
};

/* Gemma embedding scale: sqrt(2048) rounded to bf16 (the embedder multiplies in the table dtype). */
#define P5_EMBED_SCALE 45.25f
/* SigLIP attention divides q by sqrt(72) rounded to bf16 = 8.5. */
#define P5_SIG_QDIV 8.5f
/* Euler step dt = -1/num_steps; the update multiplies by dt rounded to bf16 (-0.1 -> -0.10009765625). */

/* ---- tensor kinds: one generator stream per (kind, layer) ---- */
enum p5_kind {
  /* SigLIP */
  K_SIG_STEM_W = 1, K_SIG_STEM_B, K_SIG_POSEMB,
  K_SIG_LN1_S, K_SIG_LN1_B, K_SIG_WQ, K_SIG_WK, K_SIG_WV, K_SIG_BQ, K_SIG_BK, K_SIG_BV,
  K_SIG_WO, K_SIG_BO, K_SIG_LN2_S, K_SIG_LN2_B, K_SIG_W1, K_SIG_B1, K_SIG_W2, K_SIG_B2,
  K_SIG_POST_S, K_SIG_POST_B, K_SIG_HEAD_W, K_SIG_HEAD_B,
  /* Gemma-2B prefix */
  K_GEM_EMBED = 30, K_GEM_RMS1, K_GEM_WQ, K_GEM_WK, K_GEM_WV, K_GEM_WO, K_GEM_RMS2,
  K_GEM_WG, K_GEM_WU, K_GEM_WD, K_GEM_FINAL,
  /* action expert */
  K_EXP_WQ = 50, K_EXP_WK, K_EXP_WV, K_EXP_WO, K_EXP_WG, K_EXP_WU, K_EXP_WD,
  K_EXP_ADA1_W, K_EXP_ADA1_B, K_EXP_ADA2_W, K_EXP_ADA2_B, K_EXP_FINAL_W, K_EXP_FINAL_B,
  K_AIN_W, K_AIN_B, K_AOUT_W, K_AOUT_B, K_TIN_W, K_TIN_B, K_TOUT_W, K_TOUT_B,
  /* LoRA adapters: A is [rank][in], B is [out][rank]; projection p in 0..6 = q,k,v,o,gate,up,down */
  K_LORA_GEM_A = 80, K_LORA_GEM_B = 88, K_LORA_EXP_A = 96, K_LORA_EXP_B = 104,
  /* inputs */
  K_IN_IMAGE = 120, K_IN_TOKENS, K_IN_NOISE, K_IN_KCACHE, K_IN_VCACHE, K_IN_ACTIONS,
  K_IN_TRAIN_NOISE, K_IN_TIME,
};

/* ---- generator ---- */
P5_FN uint64_t p5_mix(uint64_t z) {
  z ^= z >> 30; z *= 0xbf58476d1ce4e5b9ULL;
  z ^= z >> 27; z *= 0x94d049bb133111ebULL;
  z ^= z >> 31; return z;
}
P5_FN uint64_t p5_key(uint64_t seed, uint32_t kind, uint32_t sub) {
  return p5_mix(seed * 0x9E3779B97F4A7C15ULL ^ p5_mix(((uint64_t)kind << 32) | (uint64_t)sub));
}
P5_FN uint64_t p5_bits(uint64_t key, uint64_t ctr) {
  return p5_mix(key + ctr * 0x9E3779B97F4A7C15ULL);
}
/* Irwin-Hall(8) of 16-bit uniforms, centred: integer in [-262140, 262140], std 53509.12 */
P5_FN int32_t p5_ih8(uint64_t key, uint64_t idx) {
  uint64_t a = p5_bits(key, 2 * idx), b = p5_bits(key, 2 * idx + 1);
  int32_t s = (int32_t)(a & 0xFFFF) + (int32_t)((a >> 16) & 0xFFFF) + (int32_t)((a >> 32) & 0xFFFF) +
              (int32_t)(a >> 48) + (int32_t)(b & 0xFFFF) + (int32_t)((b >> 16) & 0xFFFF) +
              (int32_t)((b >> 32) & 0xFFFF) + (int32_t)(b >> 48);
  return s - 262140;
}
#define P5_IH8_STD 53509.12283502848
/* multiplier that turns p5_ih8 into N(0, std^2) */
static inline float p5_scale_for_std(double std) { return (float)(std / P5_IH8_STD); }

P5_FN float p5_normal(uint64_t key, uint64_t idx, float scale) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn((float)p5_ih8(key, idx), scale);
#else
  return (float)p5_ih8(key, idx) * scale;
#endif
}
P5_FN float p5_normal_off(uint64_t key, uint64_t idx, float scale, float base) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(base, __fmul_rn((float)p5_ih8(key, idx), scale));
#else
  float p = (float)p5_ih8(key, idx) * scale;
  return base + p;
#endif
}

/* bf16 round-to-nearest-even (finite inputs) */
P5_FN uint16_t p5_f2bf(float f) {
  uint32_t u;
#if defined(__CUDA_ARCH__)
  u = __float_as_uint(f);
#else
  memcpy(&u, &f, 4);
#endif
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
P5_FN float p5_bf2f(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f; memcpy(&f, &u, 4); return f;
#endif
}
P5_FN float p5_round_bf(float f) { return p5_bf2f(p5_f2bf(f)); }

/* uniform byte (images) and uniform token id */
P5_FN uint8_t p5_u8(uint64_t key, uint64_t idx) { return (uint8_t)(p5_bits(key, idx) >> 40); }
P5_FN int32_t p5_token(uint64_t key, uint64_t idx) { return (int32_t)(p5_bits(key, idx) % (uint64_t)P5_VOCAB); }

/* ---- parameter initialisation convention ----
 * Linear weights and biases: N(0, 0.02).  LoRA A/B: N(0, 0.01).
 * RMSNorm scales (used as 1+scale): N(0, 0.02).  LayerNorm scales: 1 + N(0, 0.02); LayerNorm biases N(0, 0.02).
 * Every value is rounded to bf16 before use. */
#define P5_W_STD 0.02
#define P5_LORA_STD 0.01

P5_FN int p5_kind_has_unit_base(int kind) {
  return kind == K_SIG_LN1_S || kind == K_SIG_LN2_S || kind == K_SIG_POST_S;
}

/* one parameter value (bf16 bits) */
P5_FN uint16_t p5_param_bf(uint64_t key, uint64_t idx, float scale, float base) {
  return p5_f2bf(p5_normal_off(key, idx, scale, base));
}

/* ---- host-side tables shared by the engine and the oracle (double precision, rounded once) ---- */
#include <math.h>
/* RoPE (openpi gemma._apply_rope, max_wavelength 10000, split-half pairs (i, i+128)):
 * cos/sin of pos / 10000^(2i/256) for i in [0,128).  out: [npos][128] cos then [npos][128] sin. */
static inline void p5_rope_table(int npos, float* cos_out, float* sin_out) {
  for (int p = 0; p < npos; ++p)
    for (int i = 0; i < P5_HD / 2; ++i) {
      double ts = pow(10000.0, (2.0 * i) / (double)P5_HD);
      double a = (double)p / ts;
      cos_out[(size_t)p * (P5_HD / 2) + i] = (float)cos(a);
      sin_out[(size_t)p * (P5_HD / 2) + i] = (float)sin(a);
    }
}
/* Flow-matching time schedule (openpi pi0.sample_actions): t0 = 1, t <- t + dt in fp32, dt = -1/steps. */
static inline void p5_time_schedule(int steps, float* t_out) {
  float t = 1.0f, dt = (float)(-1.0 / (double)steps);
  for (int s = 0; s < steps; ++s) { t_out[s] = t; t = t + dt; }
}
/* bf16(dt), the multiplier of the Euler update */
static inline float p5_dt_bf16(int steps) { return p5_round_bf((float)(-1.0 / (double)steps)); }
/* Sinusoidal time embedding (openpi pi0.posemb_sincos, min_period 4e-3, max_period 4.0), width w:
 * out[i] = sin(t * 2*pi / period_i), out[w/2+i] = cos(...), period_i = 4e-3 * 1000^(i/(w/2-1)). */
static inline void p5_time_embedding(float t, int w, float* out) {
  int h = w / 2;
  for (int i = 0; i < h; ++i) {
    double frac = (h > 1) ? (double)i / (double)(h - 1) : 0.0;
    double period = 4e-3 * pow(4.0 / 4e-3, frac);
    double a = (double)t * (2.0 * M_PI / period);
    out[i] = (float)sin(a);
    out[h + i] = (float)cos(a);
  }
}

#endif /* PI05_MODEL_H */

// pi05_oracle.cpp — fp32 CPU restatement of the pi0.5 inference path.  TEST INFRASTRUCTURE ONLY.
//
// Follows the model facts of the reference engine record (docs/archive/windows/π05_네이티브엔진.md:28-40)
// and the openpi functions that record cites:
//   SigLIP So400m/14            models/siglip.py:311-370   (stem in fp32, pre-LN encoder, LN eps 1e-6)
//   Gemma block / RMSNorm / RoPE models/gemma.py            (RMSNorm (1+scale), split-half RoPE, MQA)
//   pi0.5 prefix/suffix/sample  models/pi0.py:81-95,216-279 (adaRMS time conditioning, Euler dt=-0.1)
// bf16 rounding points: R() below marks every place where the bf16 JAX path stores an activation.
//
// Parity status: unpinned against the reference engine (its source and golden dumps were deleted
// from the reference repository); pinned to the rounding conventions recorded at π05_네이티브엔진.md:38-40.
#include "pi05_oracle.h"
#include "pi05_model.h"

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using std::vector;
typedef vector<float> Vf;

namespace {

struct Run {
  int flags;
  p5o_probe_fn probe;
  void* pctx;
  bool f32() const { return (flags & P5O_FP32_ACTIVATIONS) != 0; }
  float R(float x) const { return f32() ? x : p5_round_bf(x); }
  void Rv(float* x, size_t n) const {
    if (f32()) return;
    for (size_t i = 0; i < n; ++i) x[i] = p5_round_bf(x[i]);
  }
  void point(const std::string& name, const float* d, size_t n) const {
    if (probe) probe(name.c_str(), d, (int64_t)n, pctx);
  }
};

// ---------------------------------------------------------------- parameters
void gen_param(float* dst, uint64_t seed, int kind, int sub, size_t n, double stdv, float base = 0.f) {
  const uint64_t key = p5_key(seed, kind, sub);
  const float sc = p5_scale_for_std(stdv);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; ++i) dst[i] = p5_bf2f(p5_param_bf(key, (uint64_t)i, sc, base));
}
Vf param(uint64_t seed, int kind, int sub, size_t n, double stdv = P5_W_STD) {
  Vf v(n);
  gen_param(v.data(), seed, kind, sub, n, stdv, p5_kind_has_unit_base(kind) ? 1.0f : 0.0f);
  return v;
}

// ---------------------------------------------------------------- GEMM  y[M][N] = x[M][K] . W[N][K]^T
inline float hsum8(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
  lo = _mm_add_ps(lo, hi);
  lo = _mm_hadd_ps(lo, lo);
  lo = _mm_hadd_ps(lo, lo);
  return _mm_cvtss_f32(lo);
}

void gemm_nt(int M, int N, int K, const float* x, int ldx, const float* W, int ldw, float* y, int ldy) {
  const int K8 = K & ~7;
  const int nb = (N + 63) / 64, mb = (M + 63) / 64;
#pragma omp parallel for schedule(dynamic)
  for (int t = 0; t < nb * mb; ++t) {
    const int jb = (t % nb) * 64, ib = (t / nb) * 64;
    const int je = std::min(jb + 64, N), ie = std::min(ib + 64, M);
    for (int j = jb; j < je; j += 4)
      for (int i = ib; i < ie; i += 4) {
        const int ni = std::min(4, ie - i), nj = std::min(4, je - j);
        const float* xr[4];
        const float* wr[4];
        for (int a = 0; a < 4; ++a) xr[a] = x + (size_t)(i + std::min(a, ni - 1)) * ldx;
        for (int b = 0; b < 4; ++b) wr[b] = W + (size_t)(j + std::min(b, nj - 1)) * ldw;
        __m256 acc[4][4];
        for (int a = 0; a < 4; ++a)
          for (int b = 0; b < 4; ++b) acc[a][b] = _mm256_setzero_ps();
        for (int k = 0; k < K8; k += 8) {
          __m256 xv[4], wv[4];
          for (int a = 0; a < 4; ++a) xv[a] = _mm256_loadu_ps(xr[a] + k);
          for (int b = 0; b < 4; ++b) wv[b] = _mm256_loadu_ps(wr[b] + k);
          for (int a = 0; a < 4; ++a)
            for (int b = 0; b < 4; ++b) acc[a][b] = _mm256_fmadd_ps(xv[a], wv[b], acc[a][b]);
        }
        for (int a = 0; a < ni; ++a)
          for (int b = 0; b < nj; ++b) {
            float s = hsum8(acc[a][b]);
            for (int k = K8; k < K; ++k) s += xr[a][k] * wr[b][k];
            y[(size_t)(i + a) * ldy + j + b] = s;
          }
      }
  }
}

// y = R(x W^T + b)   (b may be null)
void linear(const Run& r, int M, int N, int K, const float* x, const float* W, const float* b, float* y) {
  gemm_nt(M, N, K, x, K, W, K, y, N);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)M; ++i)
    for (int j = 0; j < N; ++j) {
      float v = y[i * N + j];
      if (b) v += b[j];
      y[i * N + j] = r.R(v);
    }
}

void transpose(const float* a, int rows, int cols, int lda, float* t) {  // t[cols][rows]
#pragma omp parallel for schedule(static)
  for (int c = 0; c < cols; ++c)
    for (int rr = 0; rr < rows; ++rr) t[(size_t)c * rows + rr] = a[(size_t)rr * lda + c];
}

// ---------------------------------------------------------------- elementwise
inline float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.0f + std::tanh(c * (x + 0.044715f * x * x * x)));
}
inline float swish(float x) { return x / (1.0f + std::exp(-x)); }

// flax LayerNorm (eps 1e-6), statistics in fp32
void layernorm(const Run& r, const float* x, int T, int D, const float* s, const float* b, float* y) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* xr = x + (size_t)t * D;
    float mean = 0.f;
    for (int i = 0; i < D; ++i) mean += xr[i];
    mean /= (float)D;
    float var = 0.f;
    for (int i = 0; i < D; ++i) {
      float d = xr[i] - mean;
      var += d * d;
    }
    var /= (float)D;
    const float inv = 1.0f / std::sqrt(var + 1e-6f);
    for (int i = 0; i < D; ++i) y[(size_t)t * D + i] = r.R((xr[i] - mean) * inv * s[i] + b[i]);
  }
}

// openpi gemma.RMSNorm: normed = x / sqrt(mean(x^2) + 1e-6) in fp32;
//   plain:    normed * (1 + scale)            (1 + scale is computed in the bf16 parameter dtype)
//   adaptive: normed * (1 + scale) + shift    (scale/shift/gate come from a bf16 Dense of the time condition)
void rmsnorm(const Run& r, const float* x, int T, int D, const float* scale, const float* shift, float* y) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* xr = x + (size_t)t * D;
    float ss = 0.f;
    for (int i = 0; i < D; ++i) ss += xr[i] * xr[i];
    const float inv = 1.0f / std::sqrt(ss / (float)D + 1e-6f);
    for (int i = 0; i < D; ++i) {
      float v = xr[i] * inv * r.R(1.0f + scale[i]);
      if (shift) v += shift[i];
      y[(size_t)t * D + i] = r.R(v);
    }
  }
}

// split-half RoPE on `nheads` 256-wide heads of each row; positions pos0 + t
void rope(const Run& r, float* x, int T, int nheads, int ld, int pos0, const float* cs, const float* sn) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < nheads; ++h) {
      float* v = x + (size_t)t * ld + h * P5_HD;
      const float* c = cs + (size_t)(pos0 + t) * (P5_HD / 2);
      const float* s = sn + (size_t)(pos0 + t) * (P5_HD / 2);
      for (int i = 0; i < P5_HD / 2; ++i) {
        float x1 = v[i], x2 = v[i + P5_HD / 2];
        float a = x1 * c[i] - x2 * s[i];
        float b = x2 * c[i] + x1 * s[i];
        v[i] = r.R(a);
        v[i + P5_HD / 2] = r.R(b);
      }
    }
}

// softmax(q k^T) v for `nh` query heads of width hd.  Query head h reads key/value head
// (kv_per_head ? h : 0) (MHA vs MQA).  q already scaled.  logits and softmax in fp32,
// probabilities rounded to the activation dtype before the value product (openpi gemma.Attention).
// group > 0: queries t < group attend to the keys j < group only (two attention groups in the prefix).
void attention(const Run& r, int T, int S, int nh, int hd, const float* q, int ldq, const float* k, int ldk,
               const float* v, int ldv, bool kv_per_head, float* out, int ldo, int group = 0) {
  Vf logits((size_t)T * S), vt((size_t)hd * S), o((size_t)T * hd);
  for (int h = 0; h < nh; ++h) {
    const int kvh = kv_per_head ? h : 0;
    gemm_nt(T, S, hd, q + h * hd, ldq, k + kvh * hd, ldk, logits.data(), S);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
      float* l = logits.data() + (size_t)t * S;
      const int lim = (group > 0 && t < group) ? std::min(S, group) : S;
      float m = -INFINITY;
      for (int j = 0; j < lim; ++j) m = std::max(m, l[j]);
      float sum = 0.f;
      for (int j = 0; j < lim; ++j) {
        l[j] = std::exp(l[j] - m);
        sum += l[j];
      }
      for (int j = 0; j < lim; ++j) l[j] = r.R(l[j] / sum);
      for (int j = lim; j < S; ++j) l[j] = 0.f;
    }
    transpose(v + kvh * hd, S, hd, ldv, vt.data());
    gemm_nt(T, hd, S, logits.data(), S, vt.data(), S, o.data(), hd);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
      for (int d = 0; d < hd; ++d) out[(size_t)t * ldo + h * hd + d] = r.R(o[(size_t)t * hd + d]);
  }
}

struct Rope {
  Vf c, s;
  explicit Rope(int npos) : c((size_t)npos * P5_HD / 2), s((size_t)npos * P5_HD / 2) {
    p5_rope_table(npos, c.data(), s.data());
  }
};

// ---------------------------------------------------------------- SigLIP So400m/14
void siglip(const p5o_config* c, uint64_t seed, const uint8_t* images, float* out, const Run& r) {
  const int D = P5_SIG_W, F = P5_SIG_MLP, T = P5_SIG_TOK * c->n_cameras;
  Vf x((size_t)T * D), y((size_t)T * D), q((size_t)T * D), k((size_t)T * D), v((size_t)T * D),
      o((size_t)T * D), h((size_t)T * F);
  {
    // stem: 14x14/14 patch conv in fp32 on x = p/255*2-1, + bias + learned position embedding
    Vf patches((size_t)T * P5_SIG_K);
    for (int cam = 0; cam < c->n_cameras; ++cam)
      for (int py = 0; py < 16; ++py)
        for (int px = 0; px < 16; ++px) {
          float* pr = patches.data() + (size_t)(cam * 256 + py * 16 + px) * P5_SIG_K;
          for (int ky = 0; ky < 14; ++ky)
            for (int kx = 0; kx < 14; ++kx)
              for (int ch = 0; ch < 3; ++ch) {
                uint8_t p = images[(((size_t)cam * P5_IMG + py * 14 + ky) * P5_IMG + px * 14 + kx) * 3 + ch];
                pr[(ky * 14 + kx) * 3 + ch] = (float)p / 255.0f * 2.0f - 1.0f;
              }
        }
    Vf W = param(seed, K_SIG_STEM_W, 0, (size_t)D * P5_SIG_K), b = param(seed, K_SIG_STEM_B, 0, D),
       pe = param(seed, K_SIG_POSEMB, 0, (size_t)256 * D);
    gemm_nt(T, D, P5_SIG_K, patches.data(), P5_SIG_K, W.data(), P5_SIG_K, x.data(), D);
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < D; ++j) x[(size_t)t * D + j] = r.R(x[(size_t)t * D + j] + b[j] + pe[(size_t)(t % 256) * D + j]);
    r.point("img.stem", x.data(), x.size());
  }
  for (int l = 0; l < c->siglip_layers; ++l) {
    Vf ln1s = param(seed, K_SIG_LN1_S, l, D), ln1b = param(seed, K_SIG_LN1_B, l, D);
    Vf wq = param(seed, K_SIG_WQ, l, (size_t)D * D), wk = param(seed, K_SIG_WK, l, (size_t)D * D),
       wv = param(seed, K_SIG_WV, l, (size_t)D * D);
    Vf bq = param(seed, K_SIG_BQ, l, D), bk = param(seed, K_SIG_BK, l, D), bv = param(seed, K_SIG_BV, l, D);
    Vf wo = param(seed, K_SIG_WO, l, (size_t)D * D), bo = param(seed, K_SIG_BO, l, D);
    Vf ln2s = param(seed, K_SIG_LN2_S, l, D), ln2b = param(seed, K_SIG_LN2_B, l, D);
    Vf w1 = param(seed, K_SIG_W1, l, (size_t)F * D), b1 = param(seed, K_SIG_B1, l, F);
    Vf w2 = param(seed, K_SIG_W2, l, (size_t)D * F), b2 = param(seed, K_SIG_B2, l, D);

    layernorm(r, x.data(), T, D, ln1s.data(), ln1b.data(), y.data());
    linear(r, T, D, D, y.data(), wq.data(), bq.data(), q.data());
    linear(r, T, D, D, y.data(), wk.data(), bk.data(), k.data());
    linear(r, T, D, D, y.data(), wv.data(), bv.data(), v.data());
    for (auto& e : q) e = r.R(e / P5_SIG_QDIV);
    for (int cam = 0; cam < c->n_cameras; ++cam) {
      const size_t off = (size_t)cam * 256 * D;
      attention(r, 256, 256, P5_SIG_HEADS, P5_SIG_HD, q.data() + off, D, k.data() + off, D, v.data() + off, D,
                true, o.data() + off, D);
    }
    linear(r, T, D, D, o.data(), wo.data(), bo.data(), y.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = r.R(x[i] + y[i]);
    layernorm(r, x.data(), T, D, ln2s.data(), ln2b.data(), y.data());
    linear(r, T, F, D, y.data(), w1.data(), b1.data(), h.data());
    for (auto& e : h) e = r.R(gelu_tanh(e));
    linear(r, T, D, F, h.data(), w2.data(), b2.data(), y.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = r.R(x[i] + y[i]);
    r.point("img.l" + std::to_string(l) + ".out", x.data(), x.size());
  }
  Vf ps = param(seed, K_SIG_POST_S, 0, D), pb = param(seed, K_SIG_POST_B, 0, D);
  layernorm(r, x.data(), T, D, ps.data(), pb.data(), y.data());
  r.point("img.encoded", y.data(), y.size());
  Vf hw = param(seed, K_SIG_HEAD_W, 0, (size_t)P5_GEM_W * D), hb = param(seed, K_SIG_HEAD_B, 0, P5_GEM_W);
  linear(r, T, P5_GEM_W, D, y.data(), hw.data(), hb.data(), out);
  r.point("img.tokens", out, (size_t)T * P5_GEM_W);
}

// ---------------------------------------------------------------- Gemma-2B prefix prefill
// keys: every query attends to the first S of the P prefix tokens (S < P: a padded prompt's tail masked)
void prefill(const p5o_config* c, uint64_t seed, Vf& x, int P, float* kc, float* vc, const Run& r, int S = -1) {
  if (S < 0) S = P;
  const int D = P5_GEM_W, F = P5_GEM_MLP;
  Rope rp(P);
  Vf h((size_t)P * D), q((size_t)P * P5_QDIM), kk((size_t)P * P5_HD), vv((size_t)P * P5_HD), o((size_t)P * P5_QDIM),
      g((size_t)P * F), u((size_t)P * F), y((size_t)P * D);
  for (int l = 0; l < c->gemma_layers; ++l) {
    Vf s1 = param(seed, K_GEM_RMS1, l, D), s2 = param(seed, K_GEM_RMS2, l, D);
    Vf wq = param(seed, K_GEM_WQ, l, (size_t)P5_QDIM * D), wk = param(seed, K_GEM_WK, l, (size_t)P5_HD * D),
       wv = param(seed, K_GEM_WV, l, (size_t)P5_HD * D), wo = param(seed, K_GEM_WO, l, (size_t)D * P5_QDIM);
    rmsnorm(r, x.data(), P, D, s1.data(), nullptr, h.data());
    r.point("pre.l" + std::to_string(l) + ".norm1", h.data(), h.size());
    linear(r, P, P5_QDIM, D, h.data(), wq.data(), nullptr, q.data());
    linear(r, P, P5_HD, D, h.data(), wk.data(), nullptr, kk.data());
    linear(r, P, P5_HD, D, h.data(), wv.data(), nullptr, vv.data());
    rope(r, q.data(), P, P5_NH, P5_QDIM, 0, rp.c.data(), rp.s.data());
    rope(r, kk.data(), P, 1, P5_HD, 0, rp.c.data(), rp.s.data());
    for (auto& e : q) e *= 0.0625f;  // head_dim^-0.5, exact in bf16
    std::memcpy(kc + (size_t)l * P * P5_HD, kk.data(), kk.size() * 4);
    std::memcpy(vc + (size_t)l * P * P5_HD, vv.data(), vv.size() * 4);
    r.point("pre.l" + std::to_string(l) + ".k", kk.data(), kk.size());
    r.point("pre.l" + std::to_string(l) + ".v", vv.data(), vv.size());
    if (l == c->gemma_layers - 1) break;  // the last layer's output feeds only the unused final norm
    attention(r, P, S, P5_NH, P5_HD, q.data(), P5_QDIM, kk.data(), P5_HD, vv.data(), P5_HD, false, o.data(), P5_QDIM,
              p5o_prefix_group(r.flags));
    linear(r, P, D, P5_QDIM, o.data(), wo.data(), nullptr, y.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = r.R(x[i] + y[i]);
    wq.clear(); wq.shrink_to_fit();
    Vf wg = param(seed, K_GEM_WG, l, (size_t)F * D), wu = param(seed, K_GEM_WU, l, (size_t)F * D);
    rmsnorm(r, x.data(), P, D, s2.data(), nullptr, h.data());
    r.point("pre.l" + std::to_string(l) + ".norm2", h.data(), h.size());
    linear(r, P, F, D, h.data(), wg.data(), nullptr, g.data());
    linear(r, P, F, D, h.data(), wu.data(), nullptr, u.data());
    for (size_t i = 0; i < g.size(); ++i) g[i] = r.R(r.R(gelu_tanh(g[i])) * u[i]);
    wg.clear(); wg.shrink_to_fit(); wu.clear(); wu.shrink_to_fit();
    Vf wd = param(seed, K_GEM_WD, l, (size_t)D * F);
    linear(r, P, D, F, g.data(), wd.data(), nullptr, y.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = r.R(x[i] + y[i]);
    r.point("pre.l" + std::to_string(l) + ".out", x.data(), x.size());
  }
}

void embed_text(const p5o_config* c, uint64_t seed, const int32_t* tokens, float* out, const Run& r) {
  const uint64_t key = p5_key(seed, K_GEM_EMBED, 0);
  const float sc = p5_scale_for_std(P5_W_STD);
  for (int t = 0; t < c->n_text; ++t)
    for (int d = 0; d < P5_GEM_W; ++d) {
      float e = p5_bf2f(p5_param_bf(key, (uint64_t)tokens[t] * P5_GEM_W + d, sc, 0.f));
      out[(size_t)t * P5_GEM_W + d] = r.R(e * P5_EMBED_SCALE);
    }
}

// ---------------------------------------------------------------- action expert denoise
struct ExpertLayer {
  Vf wq, wk, wv, wo, wg, wu, wd;
};

// Soft inpainting of the PiBehavior model (π05_네이티브엔진.md:142): after an Euler step that starts above
// t_min and lands at t, the first K chunk values go back on the flow path of the known actions and the
// rest follow the Gaussian conditional through C = Sigma_UO Sigma_OO^-1.  fp32 without contraction for the
// known values, the correction summed in fp64 and rounded once.
struct Inpaint {
  int K = 0;
  float t_min = 0.f;
  const float* known = nullptr;  // [K]
  const float* corr = nullptr;   // [U][K]
};

void inpaint_step(const Inpaint& ip, const float* eps, float* x, int n, float t) {
  const int K = ip.K, U = n - K;
  const float omt = 1.0f - t;
  std::vector<float> delta(K);
  for (int k = 0; k < K; ++k) {
    const float a = t * eps[k], b = omt * ip.known[k];
    const float v = a + b;
    delta[k] = v - x[k];
    x[k] = v;
  }
  for (int u = 0; u < U; ++u) {
    double acc = 0.0;
    for (int k = 0; k < K; ++k) acc += (double)ip.corr[(size_t)u * K + k] * (double)delta[k];
    x[K + u] = x[K + u] + (float)acc;
  }
}

void denoise(const p5o_config* c, uint64_t seed, const float* kc, const float* vc, int P, const float* noise,
             float* actions, const Run& r, const Inpaint* ip = nullptr) {
  const int D = P5_EXP_W, F = P5_EXP_MLP, H = c->horizon, L = c->expert_layers, S = P + H;
  vector<ExpertLayer> W(L);
  for (int l = 0; l < L; ++l) {
    W[l].wq = param(seed, K_EXP_WQ, l, (size_t)P5_QDIM * D);
    W[l].wk = param(seed, K_EXP_WK, l, (size_t)P5_HD * D);
    W[l].wv = param(seed, K_EXP_WV, l, (size_t)P5_HD * D);
    W[l].wo = param(seed, K_EXP_WO, l, (size_t)D * P5_QDIM);
    W[l].wg = param(seed, K_EXP_WG, l, (size_t)F * D);
    W[l].wu = param(seed, K_EXP_WU, l, (size_t)F * D);
    W[l].wd = param(seed, K_EXP_WD, l, (size_t)D * F);
  }
  Vf ain_w = param(seed, K_AIN_W, 0, (size_t)D * P5_ACT_D), ain_b = param(seed, K_AIN_B, 0, D);
  Vf aout_w = param(seed, K_AOUT_W, 0, (size_t)P5_ACT_D * D), aout_b = param(seed, K_AOUT_B, 0, P5_ACT_D);
  Vf tin_w = param(seed, K_TIN_W, 0, (size_t)D * D), tin_b = param(seed, K_TIN_B, 0, D);
  Vf tout_w = param(seed, K_TOUT_W, 0, (size_t)D * D), tout_b = param(seed, K_TOUT_B, 0, D);

  // time conditioning for every step: cond = swish(Wout swish(Win emb(t) + b) + b) in fp32,
  // then one bf16 Dense per adaRMSNorm -> (scale, shift, gate)
  const int NM = 2 * L + 1;  // modulations per step: (pre-attn, pre-ffw) per layer + final
  vector<float> ts(c->num_steps);
  p5_time_schedule(c->num_steps, ts.data());
  Vf mods((size_t)c->num_steps * NM * 3 * D);
  {
    Vf emb((size_t)c->num_steps * D), c1((size_t)c->num_steps * D), cond((size_t)c->num_steps * D);
    for (int s = 0; s < c->num_steps; ++s) p5_time_embedding(ts[s], D, emb.data() + (size_t)s * D);
    Run r32 = r;
    r32.flags |= P5O_FP32_ACTIVATIONS;
    linear(r32, c->num_steps, D, D, emb.data(), tin_w.data(), tin_b.data(), c1.data());
    for (auto& e : c1) e = swish(e);
    linear(r32, c->num_steps, D, D, c1.data(), tout_w.data(), tout_b.data(), cond.data());
    for (auto& e : cond) e = r.R(swish(e));  // the bf16 Dense casts its input to bf16
    Vf out((size_t)c->num_steps * 3 * D);
    for (int m = 0; m < NM; ++m) {
      int kw = (m == NM - 1) ? K_EXP_FINAL_W : ((m & 1) ? K_EXP_ADA2_W : K_EXP_ADA1_W);
      int l = (m == NM - 1) ? 0 : m / 2;
      Vf aw = param(seed, kw, l, (size_t)3 * D * D), ab = param(seed, kw + 1, l, (size_t)3 * D);
      linear(r, c->num_steps, 3 * D, D, cond.data(), aw.data(), ab.data(), out.data());
      for (int s = 0; s < c->num_steps; ++s)
        std::memcpy(mods.data() + ((size_t)s * NM + m) * 3 * D, out.data() + (size_t)s * 3 * D, 3 * D * 4);
    }
  }
  Rope rp(S);
  const float dtb = c->num_steps > 0 ? p5_dt_bf16(c->num_steps) : 0.f;
  Vf xt(noise, noise + (size_t)H * P5_ACT_D);
  Vf x((size_t)H * D), h((size_t)H * D), q((size_t)H * P5_QDIM), o((size_t)H * P5_QDIM), y((size_t)H * D),
      g((size_t)H * F), u((size_t)H * F), v((size_t)H * P5_ACT_D);
  Vf kall((size_t)S * P5_HD), vall((size_t)S * P5_HD);
  for (int s = 0; s < c->num_steps; ++s) {
    const std::string sp = "suf.s" + std::to_string(s);
    // action_in_proj: fp32 input, bf16 weights, fp32 result; the expert casts its input to bf16
    {
      Run r32 = r;
      r32.flags |= P5O_FP32_ACTIVATIONS;
      linear(r32, H, D, P5_ACT_D, xt.data(), ain_w.data(), ain_b.data(), x.data());
      r.Rv(x.data(), x.size());
    }
    r.point(sp + ".in", x.data(), x.size());
    for (int l = 0; l < L; ++l) {
      const float* m1 = mods.data() + ((size_t)s * NM + 2 * l) * 3 * D;
      const float* m2 = mods.data() + ((size_t)s * NM + 2 * l + 1) * 3 * D;
      rmsnorm(r, x.data(), H, D, m1, m1 + D, h.data());
      linear(r, H, P5_QDIM, D, h.data(), W[l].wq.data(), nullptr, q.data());
      std::memcpy(kall.data(), kc + (size_t)l * P * P5_HD, (size_t)P * P5_HD * 4);
      std::memcpy(vall.data(), vc + (size_t)l * P * P5_HD, (size_t)P * P5_HD * 4);
      linear(r, H, P5_HD, D, h.data(), W[l].wk.data(), nullptr, kall.data() + (size_t)P * P5_HD);
      linear(r, H, P5_HD, D, h.data(), W[l].wv.data(), nullptr, vall.data() + (size_t)P * P5_HD);
      rope(r, q.data(), H, P5_NH, P5_QDIM, P, rp.c.data(), rp.s.data());
      rope(r, kall.data() + (size_t)P * P5_HD, H, 1, P5_HD, P, rp.c.data(), rp.s.data());
      for (auto& e : q) e *= 0.0625f;
      attention(r, H, S, P5_NH, P5_HD, q.data(), P5_QDIM, kall.data(), P5_HD, vall.data(), P5_HD, false, o.data(),
                P5_QDIM);
      linear(r, H, D, P5_QDIM, o.data(), W[l].wo.data(), nullptr, y.data());
      for (int t = 0; t < H; ++t)
        for (int j = 0; j < D; ++j) {
          size_t i = (size_t)t * D + j;
          x[i] = r.R(x[i] + r.R(y[i] * m1[2 * D + j]));
        }
      rmsnorm(r, x.data(), H, D, m2, m2 + D, h.data());
      linear(r, H, F, D, h.data(), W[l].wg.data(), nullptr, g.data());
      linear(r, H, F, D, h.data(), W[l].wu.data(), nullptr, u.data());
      for (size_t i = 0; i < g.size(); ++i) g[i] = r.R(r.R(gelu_tanh(g[i])) * u[i]);
      linear(r, H, D, F, g.data(), W[l].wd.data(), nullptr, y.data());
      for (int t = 0; t < H; ++t)
        for (int j = 0; j < D; ++j) {
          size_t i = (size_t)t * D + j;
          x[i] = r.R(x[i] + r.R(y[i] * m2[2 * D + j]));
        }
      r.point(sp + ".l" + std::to_string(l) + ".out", x.data(), x.size());
    }
    const float* mf = mods.data() + ((size_t)s * NM + NM - 1) * 3 * D;
    rmsnorm(r, x.data(), H, D, mf, mf + D, h.data());
    r.point(sp + ".final", h.data(), h.size());
    linear(r, H, P5_ACT_D, D, h.data(), aout_w.data(), aout_b.data(), v.data());
    r.point(sp + ".v", v.data(), v.size());
    for (size_t i = 0; i < xt.size(); ++i) xt[i] = xt[i] + r.R(dtb * v[i]);
    if (ip && ip->K > 0 && ts[s] > ip->t_min) {
      // the time after step s, accumulated in fp32 as the schedule is
      const float dt = (float)(-1.0 / (double)c->num_steps);
      float t = 1.0f;
      for (int q = 0; q <= s; ++q) t = t + dt;
      inpaint_step(*ip, noise, xt.data(), (int)xt.size(), t);
    }
    r.point(sp + ".x", xt.data(), xt.size());
  }
  std::memcpy(actions, xt.data(), xt.size() * 4);
}

bool check(const p5o_config* c) {
  return c && c->siglip_layers >= 0 && c->gemma_layers >= 1 && c->expert_layers == c->gemma_layers &&
         c->num_steps >= 1 && c->n_cameras >= 1 && c->n_text >= 0 && c->horizon >= 1;
}

}  // namespace

extern "C" {

int p5o_threads(void) { return omp_get_max_threads(); }

// synthetic workload (same generator streams as the engine's pi05_synth_* helpers)
void p5o_gen_images(uint64_t seed, int sample, int n_cam, uint8_t* out) {
  const uint64_t key = p5_key(seed, K_IN_IMAGE, (uint32_t)sample);
  const int64_t n = (int64_t)n_cam * P5_IMG * P5_IMG * 3;
  for (int64_t i = 0; i < n; ++i) out[i] = p5_u8(key, (uint64_t)i);
}
void p5o_gen_tokens(uint64_t seed, int sample, int n, int32_t* out) {
  const uint64_t key = p5_key(seed, K_IN_TOKENS, (uint32_t)sample);
  for (int i = 0; i < n; ++i) out[i] = p5_token(key, (uint64_t)i);
}
void p5o_gen_normal(uint64_t seed, int kind, int sub, int64_t n, double stdv, int round_bf16, float* out) {
  const uint64_t key = p5_key(seed, kind, (uint32_t)sub);
  const float sc = p5_scale_for_std(stdv);
  for (int64_t i = 0; i < n; ++i) {
    float v = p5_normal(key, (uint64_t)i, sc);
    out[i] = round_bf16 ? p5_round_bf(v) : v;
  }
}
void p5o_gen_param(uint64_t seed, int kind, int sub, int64_t n, double stdv, float* out) {
  gen_param(out, seed, kind, sub, (size_t)n, stdv, p5_kind_has_unit_base(kind) ? 1.0f : 0.0f);
}
void p5o_gen_param_at(uint64_t seed, int kind, int sub, int64_t first, int64_t n, double stdv, float* out) {
  const uint64_t key = p5_key(seed, kind, sub);
  const float sc = p5_scale_for_std(stdv), base = p5_kind_has_unit_base(kind) ? 1.0f : 0.0f;
  for (int64_t i = 0; i < n; ++i) out[i] = p5_bf2f(p5_param_bf(key, (uint64_t)(first + i), sc, base));
}

int p5o_siglip(const p5o_config* c, uint64_t seed, const uint8_t* images, float* img_tokens, int flags,
               p5o_probe_fn probe, void* ctx) {
  if (!check(c)) return -1;
  Run r{flags, probe, ctx};
  siglip(c, seed, images, img_tokens, r);
  return 0;
}

int p5o_prefill_embedded(const p5o_config* c, uint64_t seed, const float* prefix_emb, int P, float* kcache,
                         float* vcache, int flags, p5o_probe_fn probe, void* ctx) {
  if (!check(c) || P < 1) return -1;
  Run r{flags, probe, ctx};
  Vf x(prefix_emb, prefix_emb + (size_t)P * P5_GEM_W);
  prefill(c, seed, x, P, kcache, vcache, r);
  return 0;
}

int p5o_prefix_embed(const p5o_config* c, uint64_t seed, const uint8_t* images, const int32_t* tokens, float* out,
                     int flags) {
  if (!check(c)) return -1;
  Run r{flags, nullptr, nullptr};
  siglip(c, seed, images, out, r);
  embed_text(c, seed, tokens, out + (size_t)P5_SIG_TOK * c->n_cameras * P5_GEM_W, r);
  return 0;
}

int p5o_valid_prefix(const p5o_config* c, const int32_t* tokens, int flags) {
  const int P = P5_SIG_TOK * c->n_cameras + c->n_text;
  if (!(flags & P5O_TEXT_PAD_MASK)) return P;
  int len = c->n_text;  // openpi pads prompts with id 0 and masks the padding
  while (len > 1 && tokens[len - 1] == 0) --len;
  return P5_SIG_TOK * c->n_cameras + len;
}

int p5o_prefill(const p5o_config* c, uint64_t seed, const uint8_t* images, const int32_t* tokens, float* kcache,
                float* vcache, int flags, p5o_probe_fn probe, void* ctx) {
  if (!check(c)) return -1;
  Run r{flags, probe, ctx};
  const int P = P5_SIG_TOK * c->n_cameras + c->n_text;
  Vf x((size_t)P * P5_GEM_W);
  siglip(c, seed, images, x.data(), r);
  embed_text(c, seed, tokens, x.data() + (size_t)P5_SIG_TOK * c->n_cameras * P5_GEM_W, r);
  r.point("txt.emb", x.data() + (size_t)P5_SIG_TOK * c->n_cameras * P5_GEM_W, (size_t)c->n_text * P5_GEM_W);
  prefill(c, seed, x, P, kcache, vcache, r, p5o_valid_prefix(c, tokens, flags));
  return 0;
}

int p5o_denoise(const p5o_config* c, uint64_t seed, const float* kcache, const float* vcache, int P,
                const float* noise, float* actions, int flags, p5o_probe_fn probe, void* ctx) {
  if (!check(c) || P < 1) return -1;
  Run r{flags, probe, ctx};
  denoise(c, seed, kcache, vcache, P, noise, actions, r);
  return 0;
}

int p5o_denoise_inpaint(const p5o_config* c, uint64_t seed, const float* kcache, const float* vcache, int P,
                        const float* noise, float* actions, int flags, int fixed, float t_min, const float* known,
                        const float* corr) {
  if (!check(c) || P < 1 || fixed < 0 || fixed >= c->horizon || (fixed > 0 && (!known || !corr))) return -1;
  Run r{flags, nullptr, nullptr};
  Inpaint ip;
  ip.K = fixed * P5_ACT_D;
  ip.t_min = t_min;
  ip.known = known;
  ip.corr = corr;
  denoise(c, seed, kcache, vcache, P, noise, actions, r, &ip);
  return 0;
}

}  // extern "C"

// train.cuh — LoRA train step of the pi0.5 engine (included by engine.cu; shares its helpers).
//
// Replaces the reference's LoraTrainer::accumulate / finalize_grads / opt_step (π05_네이티브엔진.md:215,
// :226-229).  Per sample: t ~ Beta(1.5,1)*0.999+0.001 (drawn by the caller), x_t = t*eps + (1-t)*a,
// u = eps - a, v = net(x_t, t, prefix), loss = mean((v-u)^2) (openpi pi0.py:189-214).  Trainable: rank-16
// LoRA (scale alpha/r = 2) on q/k/v/o/gate/up/down of the Gemma-2B prefix and of the action expert;
// SigLIP, embeddings, norms and projections are frozen.
//
// Every LoRA projection is one tcgen05 GEMM in each direction.  Forward: the input buffer carries
// 16 extra columns per adapter holding 2*R(x A^T) and the weight carries B^T in the matching columns:
//   y = [x | 2U] . [W | B]^T = x W^T + 2 (x A^T) B^T.
// Backward: dx = [dy | 2V] . [W^T | A^T]^T with V = R(dy B) and a transposed copy of the frozen
// weight; dB = dy^T (2U) and dA = (2V)^T x reduce over tokens and read dy / x MN-major.
// Activations of every layer are kept (B200 has the memory), so nothing is recomputed.
#pragma once
#include "attention_bwd.cuh"
#include "attention_bwd_tc.cuh"
#include "attention_bwd_dq_pipe.cuh"
#include "train_kernels.cuh"
#include "dp_nccl.cuh"

namespace {

struct LoraGroup {
  int n_ad = 1, K = 0, F = 0, mode = 0;  // adapters sharing the input; input width; base output rows
  int Fa[3] = {0, 0, 0};                 // output rows per adapter
  long offA[3] = {0, 0, 0}, offB[3] = {0, 0, 0};
  bf16 *Wf = nullptr, *Wb = nullptr, *Acat = nullptr, *Btcat = nullptr;
  int ldf() const { return K + 16 * n_ad; }
  int ldb() const { return F + 16 * n_ad; }
};
struct TrainLayer {
  LoraGroup qkv, o, gu, dn;
};
struct Saved {  // one stack (prefix or suffix), one layer
  bf16 *xin, *h1, *qkv, *o, *xmid, *h2, *gu, *act;
  bf16 *uT_qkv, *uT_o, *uT_gu, *uT_dn;
  float* lse;
};

}  // namespace

struct Trainer {
  pi05_lora_config cfg;
  int mb = 8;
  int n_total = 0;  // samples in the current optimizer step (loss normalisation)
  int n_seen = 0;   // samples accumulated since the last zero_grads: the buffer holds their mean
  // data parallelism (pi05_lora_attach_nccl): `overlap` averages each layer's gradients over the ranks as
  // soon as the backward pass of the current (last) micro-batch has finished that layer; `reduced` says
  // the buffer already holds the average of the ranks
  struct DpComm* dp = nullptr;
  bool overlap = false, reduced = false;
  long n_params = 0;
  float *p = nullptr, *g = nullptr, *m = nullptr, *v = nullptr;
  float* ema = nullptr;  // EMA of p (cfg.ema_decay > 0)
  float* sumsq = nullptr;
  int step = 0;
  std::vector<TrainLayer> gl, el;
  std::vector<Saved> sp, ss;
  bf16* xin_p_final = nullptr;  // prefix output of the last layer (unused) is not kept
  bf16* xin_s_final = nullptr;
  // per micro-batch
  float *d_t, *d_eps, *d_act, *d_xt, *d_u, *d_dv, *d_rowloss, *d_loss;
  float *d_temb, *d_c1, *d_c2;
  bf16 *d_cond, *mods;
  bf16 *hf;
  // backward workspaces
  float *gx_p, *gx_s, *Dp, *Ds;
  bf16 *dy_p, *dy_s, *dact_p, *dact_s, *dgu_p, *dgu_s, *dh_p, *dh_s, *do_p, *do_s, *dqkv_p, *dqkv_s, *vT;
  // fp32 query-split partials of the tensor-core dK / dV kernels: [mb][key blocks][splits][128][256]
  float* dkv_ws = nullptr;
  size_t dkv_ws_rows = 0;  // capacity in 256-float rows
};

namespace {

// ------------------------------------------------------------------ parameter layout
void lora_group_layout(LoraGroup& G, int n_ad, int K, int F, int mode, const int* Fa, long& off) {
  G.n_ad = n_ad;
  G.K = K;
  G.F = F;
  G.mode = mode;
  for (int a = 0; a < n_ad; ++a) {
    G.Fa[a] = Fa[a];
    G.offA[a] = off;
    off += 16L * K;
    G.offB[a] = off;
    off += (long)Fa[a] * 16;
  }
}

void lora_layout(pi05_engine* e, Trainer* T) {
  long off = 0;
  const int L = e->cfg.gemma_layers;
  T->gl.resize(L);
  T->el.resize(L);
  for (int s = 0; s < 2; ++s)
    for (int l = 0; l < L; ++l) {
      TrainLayer& t = s == 0 ? T->gl[l] : T->el[l];
      const int D = s == 0 ? P5_GEM_W : P5_EXP_W, F = s == 0 ? P5_GEM_MLP : P5_EXP_MLP;
      const int fq[3] = {P5_QDIM, P5_HD, P5_HD}, fo[1] = {D}, fgu[2] = {F, F}, fd[1] = {D};
      lora_group_layout(t.qkv, 3, D, P5_QKV, 1, fq, off);
      lora_group_layout(t.o, 1, P5_QDIM, D, 0, fo, off);
      lora_group_layout(t.gu, 2, D, 2 * F, 2, fgu, off);
      lora_group_layout(t.dn, 1, F, D, 0, fd, off);
    }
  T->n_params = off;
}

bool talloc(pi05_engine* e, void** p, size_t bytes) { return dalloc(e, p, bytes); }

// dQ of the attention backward for the query segment a.qs of nb batch items: the tcgen05 kernel
// (attention_bwd_tc.cuh), or the mma.sync one when PI05_ATTN_TC=0.
bool attn_bwd_dq(pi05_engine* e, const AttnBwdArgs& a, int nb) {
  const int rows = a.qs.T * P5_NH;
  if (!e->attn_tc)
    return launch(e, attn_bwd_dq_kernel, dim3((rows + 63) / 64, 1, nb), dim3(128), (size_t)ABW_SMEM_DQ, false, a);
  using C = AttnBwdTcCfg;
  CUtensorMap tq, tdo, tk1, tv1, tk2, tv2;
  auto row_map = [&](CUtensorMap* m, const bf16* base, int ld, long bstride) {
    const uint64_t dims[4] = {P5_HD, 8, (uint64_t)a.qs.T, (uint64_t)nb};
    const uint64_t st[3] = {P5_HD * 2, (uint64_t)ld * 2, (uint64_t)bstride * 2};
    const uint32_t box[4] = {64, 8, 16, 1};
    return make_tmap_nd(e, m, base, 4, dims, st, box);
  };
  auto kv_map = [&](CUtensorMap* m, const bf16* base, int len, int ld, long bstride) {
    const uint64_t dims[3] = {P5_HD, (uint64_t)len, (uint64_t)nb};
    const uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)bstride * 2};
    const uint32_t box[3] = {64, C::KT, 1};
    return make_tmap_nd(e, m, base, 3, dims, st, box);
  };
  if (!row_map(&tq, a.qs.q, a.qs.ldq, a.qs.qb) || !row_map(&tdo, a.qs.dO, a.qs.ldo, a.qs.ob)) return false;
  if (!kv_map(&tk1, a.k1, a.len1, a.ld1, a.b1stride) || !kv_map(&tv1, a.v1, a.len1, a.ld1, a.b1stride)) return false;
  if (a.len2 > 0) {
    if (!kv_map(&tk2, a.k2, a.len2, a.ld2, a.b2stride) || !kv_map(&tv2, a.v2, a.len2, a.ld2, a.b2stride)) return false;
  } else {
    tk2 = tk1;
    tv2 = tv1;
  }
  if ((a.ld_dq * 2) % 16 || (a.dq_b * 2) % 16 || ((uintptr_t)a.dq & 15))
    return set_err(e, "attention backward: dq rows must be 16-byte aligned");
  if (e->attn_bwd_pipe)
    return launch(e, attn_bwd_dq_pipe_kernel, dim3((rows + AttnBwdPipeCfg::ROWS - 1) / AttnBwdPipeCfg::ROWS, 1, nb),
                  dim3(384), (size_t)AttnBwdPipeCfg::SMEM, false, tq, tdo, tk1, tv1, tk2, tv2, a, e->d_status);
  return launch(e, attn_bwd_dq_tc_kernel, dim3((rows + C::ROWS - 1) / C::ROWS, 1, nb), dim3(384), (size_t)C::SMEM, false,
                tq, tdo, tk1, tv1, tk2, tv2, a, e->d_status);
}

// dK and dV of the keys of segment a.kseg against the query segments a.qa (and a.qbseg), for nb batch
// items: the tcgen05 kernels (query tiles split over CTAs so that ~2 waves of CTAs run, partials
// summed by attn_bwd_dkv_reduce_kernel), or the mma.sync ones when PI05_ATTN_TC=0.
bool attn_bwd_dkv(pi05_engine* e, Trainer* T, const AttnBwdArgs& a, int nb) {
  const int seg_len = a.kseg == 1 ? a.len1 : a.len2;
  if (!e->attn_tc) {
    const dim3 g((seg_len + 63) / 64, 1, nb);
    return launch(e, attn_bwd_dkv_kernel<true>, g, dim3(128), (size_t)ABW_SMEM_DKV, false, a) &&
           launch(e, attn_bwd_dkv_kernel<false>, g, dim3(128), (size_t)ABW_SMEM_DKV, false, a);
  }
  using C = AttnBwdKvCfg;
  CUtensorMap tk, tv, tqa, tdoa, tqb, tdob;
  auto key_map = [&](CUtensorMap* m, const bf16* base, int ld, long bstride) {
    const uint64_t dims[3] = {P5_HD, (uint64_t)seg_len, (uint64_t)nb};
    const uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)bstride * 2};
    const uint32_t box[3] = {64, C::KEYS, 1};
    return make_tmap_nd(e, m, base, 3, dims, st, box);
  };
  auto row_map = [&](CUtensorMap* m, const QSeg& q, bool dO) {
    const uint64_t dims[4] = {P5_HD, 8, (uint64_t)q.T, (uint64_t)nb};
    const uint64_t st[3] = {P5_HD * 2, (uint64_t)(dO ? q.ldo : q.ldq) * 2, (uint64_t)(dO ? q.ob : q.qb) * 2};
    const uint32_t box[4] = {64, 8, 8, 1};  // 8 tokens x 8 heads = one 64-row query tile
    return make_tmap_nd(e, m, dO ? q.dO : q.q, 4, dims, st, box);
  };
  const bf16* kb = a.kseg == 1 ? a.k1 : a.k2;
  const bf16* vb = a.kseg == 1 ? a.v1 : a.v2;
  const int ld = a.kseg == 1 ? a.ld1 : a.ld2;
  const long bs = a.kseg == 1 ? a.b1stride : a.b2stride;
  if (!key_map(&tk, kb, ld, bs) || !key_map(&tv, vb, ld, bs) || !row_map(&tqa, a.qa, false) ||
      !row_map(&tdoa, a.qa, true))
    return false;
  if (a.nq > 1) {
    if (!row_map(&tqb, a.qbseg, false) || !row_map(&tdob, a.qbseg, true)) return false;
  } else {
    tqb = tqa;
    tdob = tdoa;
  }
  if ((a.ld_dkv * 2) % 16 || (a.dkv_b * 2) % 16 || ((uintptr_t)a.dk & 15) || ((uintptr_t)a.dv & 15))
    return set_err(e, "attention backward: dk / dv rows must be 16-byte aligned");
  const int kblocks = (seg_len + C::KEYS - 1) / C::KEYS;
  const int nt = (a.qa.T + 7) / 8 + (a.nq > 1 ? (a.qbseg.T + 7) / 8 : 0);
  int splits = std::max(1, (2 * e->num_sms + kblocks * nb - 1) / (kblocks * nb));
  splits = std::min(std::min(splits, (int)ABW_KV_MAX_SPLITS), std::max(1, nt / 4));
  while (splits > 1 && (size_t)nb * kblocks * splits * C::KEYS > T->dkv_ws_rows) --splits;
  const dim3 grid(kblocks, splits, nb);
  for (int dk = 1; dk >= 0; --dk) {
    const size_t sp = (size_t)AttnBwdKvPipeCfg::SMEM;
    const bool ok =
        e->attn_bwd_pipe
            ? (dk ? launch(e, attn_bwd_dkv_pipe_kernel<true>, grid, dim3(384), sp, false, tk, tv, tqa, tdoa, tqb, tdob,
                           a, T->dkv_ws, e->d_status)
                  : launch(e, attn_bwd_dkv_pipe_kernel<false>, grid, dim3(384), sp, false, tk, tv, tqa, tdoa, tqb,
                           tdob, a, T->dkv_ws, e->d_status))
        : dk ? launch(e, attn_bwd_dkv_tc_kernel<true>, grid, dim3(384), (size_t)C::SMEM, false, tk, tv, tqa, tdoa, tqb,
                      tdob, a, T->dkv_ws, e->d_status)
             : launch(e, attn_bwd_dkv_tc_kernel<false>, grid, dim3(384), (size_t)C::SMEM, false, tk, tv, tqa, tdoa, tqb,
                      tdob, a, T->dkv_ws, e->d_status);
    if (!ok) return false;
    if (splits > 1) {
      const long n = (long)nb * seg_len * 32;
      if (!launch(e, attn_bwd_dkv_reduce_kernel, dim3((n + 255) / 256), dim3(256), 0, false, (const float*)T->dkv_ws,
                  kblocks, splits, seg_len, nb, dk ? a.dk : a.dv, a.ld_dkv, a.dkv_b))
        return false;
    }
  }
  return true;
}
// token-major transposes ([16n][R]) are TMA operands: rows padded to 16 bytes
inline long pad8(long r) { return (r + 7) & ~7L; }

bool alloc_group(pi05_engine* e, LoraGroup& G, const bf16* W) {
  if (!talloc(e, (void**)&G.Wf, (size_t)G.F * G.ldf() * 2) || !talloc(e, (void**)&G.Wb, (size_t)G.K * G.ldb() * 2) ||
      !talloc(e, (void**)&G.Acat, (size_t)16 * G.n_ad * G.K * 2) ||
      !talloc(e, (void**)&G.Btcat, (size_t)16 * G.n_ad * G.F * 2))
    return false;
  lora_frozen_copy_kernel<<<148 * 8, 256, 0, e->stream>>>(W, G.F, G.K, G.Wf, G.ldf(), G.Wb, G.ldb());
  CK(cudaGetLastError());
  return true;
}

bool scatter_group(pi05_engine* e, Trainer* T, const LoraGroup& G) {
  for (int a = 0; a < G.n_ad; ++a) {
    LoraScatter s;
    s.A = T->p + G.offA[a];
    s.B = T->p + G.offB[a];
    s.K = G.K;
    s.Fa = G.Fa[a];
    s.Wf = G.Wf;
    s.ld_wf = G.ldf();
    s.colB = G.K + 16 * a;
    s.row_off = G.mode == 1 ? (a == 0 ? 0 : (a == 1 ? P5_QDIM : P5_QDIM + P5_HD)) : (G.mode == 2 ? a : 0);
    s.row_step = G.mode == 2 ? 2 : 1;
    s.Wb = G.Wb;
    s.ld_wb = G.ldb();
    s.colA = G.F + 16 * a;
    s.Acat = G.Acat;
    s.Btcat = G.Btcat;
    s.ld_bt = G.F;
    s.arow = 16 * a;
    lora_scatter_kernel<<<148 * 4, 256, 0, e->stream>>>(s);
    CK(cudaGetLastError());
  }
  return true;
}

bool scatter_all(pi05_engine* e, Trainer* T) {
  for (int s = 0; s < 2; ++s)
    for (TrainLayer& t : (s == 0 ? T->gl : T->el))
      if (!scatter_group(e, T, t.qkv) || !scatter_group(e, T, t.o) || !scatter_group(e, T, t.gu) ||
          !scatter_group(e, T, t.dn))
        return false;
  return true;
}

bool lora_create(pi05_engine* e, const pi05_lora_config* c, uint64_t seed) {
  Trainer* T = new Trainer();
  e->tr = T;
  T->cfg = *c;
  T->mb = c->micro_batch;
  if (T->mb > e->max_batch) return set_err(e, "lora: micro_batch exceeds the engine's max_batch");
  lora_layout(e, T);
  const int L = e->cfg.gemma_layers, P = e->P, H = e->cfg.horizon, mb = T->mb;
  const long np = T->n_params;
  if (!talloc(e, (void**)&T->p, np * 4) || !talloc(e, (void**)&T->g, np * 4) || !talloc(e, (void**)&T->m, np * 4) ||
      !talloc(e, (void**)&T->v, np * 4) || !talloc(e, (void**)&T->sumsq, 1024 * 4))
    return false;
  if (c->ema_decay > 0.f && !talloc(e, (void**)&T->ema, np * 4)) return false;
  lora_init_kernel<<<148 * 8, 256, 0, e->stream>>>(T->p, np, p5_key(seed, K_LORA_GEM_A, 0),
                                                    p5_scale_for_std(P5_LORA_STD));
  CK(cudaGetLastError());
  if (T->ema) CK(cudaMemcpyAsync(T->ema, T->p, np * 4, cudaMemcpyDeviceToDevice, e->stream));  // EMA starts at p
  for (int l = 0; l < L; ++l) {
    const GemLayer& g = e->gem[l];
    const ExpLayer& x = e->ex[l];
    if (!alloc_group(e, T->gl[l].qkv, g.wqkv) || !alloc_group(e, T->gl[l].o, g.wo) ||
        !alloc_group(e, T->gl[l].gu, g.wgu) || !alloc_group(e, T->gl[l].dn, g.wd) ||
        !alloc_group(e, T->el[l].qkv, x.wqkv) || !alloc_group(e, T->el[l].o, x.wo) ||
        !alloc_group(e, T->el[l].gu, x.wgu) || !alloc_group(e, T->el[l].dn, x.wd))
      return false;
  }
  if (!scatter_all(e, T)) return false;
  // saved activations
  const long Rp = (long)mb * P, Rs = (long)mb * H;
  T->sp.resize(L);
  T->ss.resize(L);
  for (int s = 0; s < 2; ++s)
    for (int l = 0; l < L; ++l) {
      Saved& S = s == 0 ? T->sp[l] : T->ss[l];
      const long R = s == 0 ? Rp : Rs;
      const int D = s == 0 ? P5_GEM_W : P5_EXP_W, F = s == 0 ? P5_GEM_MLP : P5_EXP_MLP;
      if (!talloc(e, (void**)&S.xin, R * D * 2) || !talloc(e, (void**)&S.h1, R * (D + 48) * 2) ||
          !talloc(e, (void**)&S.qkv, R * P5_QKV * 2) || !talloc(e, (void**)&S.o, R * (P5_QDIM + 16) * 2) ||
          !talloc(e, (void**)&S.xmid, R * D * 2) || !talloc(e, (void**)&S.h2, R * (D + 32) * 2) ||
          !talloc(e, (void**)&S.gu, R * 2 * F * 2) || !talloc(e, (void**)&S.act, R * (F + 16) * 2) ||
          !talloc(e, (void**)&S.uT_qkv, 48 * pad8(R) * 2) || !talloc(e, (void**)&S.uT_o, 16 * pad8(R) * 2) ||
          !talloc(e, (void**)&S.uT_gu, 32 * pad8(R) * 2) || !talloc(e, (void**)&S.uT_dn, 16 * pad8(R) * 2) ||
          !talloc(e, (void**)&S.lse, R * P5_NH * 4))
        return false;
    }
  if (!talloc(e, (void**)&T->xin_p_final, Rp * P5_GEM_W * 2) || !talloc(e, (void**)&T->xin_s_final, Rs * P5_EXP_W * 2))
    return false;
  const size_t actb = (size_t)Rs * P5_ACT_D * 4;
  if (!talloc(e, (void**)&T->d_t, 1024 * 4) || !talloc(e, (void**)&T->d_eps, actb) ||
      !talloc(e, (void**)&T->d_act, actb) || !talloc(e, (void**)&T->d_xt, actb) || !talloc(e, (void**)&T->d_u, actb) ||
      !talloc(e, (void**)&T->d_dv, actb) || !talloc(e, (void**)&T->d_rowloss, Rs * 4) ||
      !talloc(e, (void**)&T->d_loss, 64) || !talloc(e, (void**)&T->d_temb, (size_t)mb * P5_EXP_W * 4) ||
      !talloc(e, (void**)&T->d_c1, (size_t)mb * P5_EXP_W * 4) || !talloc(e, (void**)&T->d_c2, (size_t)mb * P5_EXP_W * 4) ||
      !talloc(e, (void**)&T->d_cond, (size_t)mb * P5_EXP_W * 2) ||
      !talloc(e, (void**)&T->mods, (size_t)mb * e->NM * 3 * P5_EXP_W * 2) ||
      !talloc(e, (void**)&T->hf, Rs * P5_EXP_W * 2))
    return false;
  // backward workspaces
  if (!talloc(e, (void**)&T->gx_p, Rp * P5_GEM_W * 4) || !talloc(e, (void**)&T->gx_s, Rs * P5_EXP_W * 4) ||
      !talloc(e, (void**)&T->Dp, Rp * P5_NH * 4) || !talloc(e, (void**)&T->Ds, Rs * P5_NH * 4) ||
      !talloc(e, (void**)&T->dy_p, Rp * (P5_GEM_W + 16) * 2) || !talloc(e, (void**)&T->dy_s, Rs * (P5_EXP_W + 16) * 2) ||
      !talloc(e, (void**)&T->dact_p, Rp * P5_GEM_MLP * 2) || !talloc(e, (void**)&T->dact_s, Rs * P5_EXP_MLP * 2) ||
      !talloc(e, (void**)&T->dgu_p, Rp * (2 * P5_GEM_MLP + 32) * 2) ||
      !talloc(e, (void**)&T->dgu_s, Rs * (2 * P5_EXP_MLP + 32) * 2) || !talloc(e, (void**)&T->dh_p, Rp * P5_GEM_W * 2) ||
      !talloc(e, (void**)&T->dh_s, Rs * P5_EXP_W * 2) || !talloc(e, (void**)&T->do_p, Rp * P5_QDIM * 2) ||
      !talloc(e, (void**)&T->do_s, Rs * P5_QDIM * 2) || !talloc(e, (void**)&T->dqkv_p, Rp * (P5_QKV + 48) * 2) ||
      !talloc(e, (void**)&T->dqkv_s, Rs * (P5_QKV + 48) * 2) || !talloc(e, (void**)&T->vT, 48 * pad8(std::max(Rp, Rs)) * 2))
    return false;
  T->dkv_ws_rows = (size_t)mb * ((P + AttnBwdKvCfg::KEYS - 1) / AttnBwdKvCfg::KEYS) * ABW_KV_MAX_SPLITS * AttnBwdKvCfg::KEYS;
  if (!talloc(e, (void**)&T->dkv_ws, T->dkv_ws_rows * P5_HD * 4)) return false;
  CK(cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ABW_SMEM_DQ));
  CK(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnBwdTcCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dq_pipe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnBwdPipeCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_pipe_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnBwdKvPipeCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_pipe_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnBwdKvPipeCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnBwdKvCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnBwdKvCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ABW_SMEM_DKV));
  CK(cudaFuncSetAttribute(attn_bwd_dkv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ABW_SMEM_DKV));
  CK(cudaStreamSynchronize(e->stream));
  return true;
}

// ------------------------------------------------------------------ GEMM helpers of the LoRA path
// U = R(x A^T) * 2 into the extra columns of the input buffer, and its transpose [16n][R]
bool lora_u(pi05_engine* e, const LoraGroup& G, bf16* xcat, int R, bf16* uT) {
  Lin L{xcat, G.ldf(), R, G.Acat, G.K, 16 * G.n_ad, G.K};
  L.epi = EPI_STORE_T;
  L.no_swap = true;
  L.out = xcat + G.K;
  L.ld_out = G.ldf();
  L.out_scale = 2.0f;
  L.out_t = uT;
  L.ld_out_t = (int)pad8(R);
  return linear(e, L);
}
// V = R(dy B) * 2 into the extra columns of the gradient buffer, and its transpose
bool lora_v(pi05_engine* e, const LoraGroup& G, bf16* dycat, int R, bf16* vT) {
  Lin L{dycat, G.ldb(), R, G.Btcat, G.F, 16 * G.n_ad, G.F};
  L.epi = EPI_STORE_T;
  L.no_swap = true;
  L.out = dycat + G.F;
  L.ld_out = G.ldb();
  L.out_scale = 2.0f;
  L.out_t = vT;
  L.ld_out_t = (int)pad8(R);
  return linear(e, L);
}
// dB_a += dy^T (2U) over the adapter's rows; dA_a += (2V)^T x
bool lora_wgrad(pi05_engine* e, Trainer* T, const LoraGroup& G, const bf16* dycat, const bf16* xcat, const bf16* uT,
                const bf16* vT, int R) {
  Lin b{dycat, G.ldb(), G.F, uT, (int)pad8(R), 16 * G.n_ad, R};
  b.amn = true;
  b.epi = EPI_LORA_GRAD;
  b.out_f32 = T->g;
  b.lg_mode = G.mode;
  b.lg_trans = 0;
  for (int a = 0; a < 3; ++a) b.lg_off[a] = G.offB[a];
  if (!linear(e, b)) return false;
  Lin a{xcat, G.ldf(), G.K, vT, (int)pad8(R), 16 * G.n_ad, R};
  a.amn = true;
  a.epi = EPI_LORA_GRAD;
  a.out_f32 = T->g;
  a.lg_trans = 1;
  a.lg_K = G.K;
  for (int i = 0; i < 3; ++i) a.lg_off[i] = G.offA[i];
  return linear(e, a);
}
// dx = [dy | 2V] . [W^T | A^T]^T
bool lora_dx(pi05_engine* e, const LoraGroup& G, const bf16* dycat, int R, bf16* dx) {
  Lin L{dycat, G.ldb(), R, G.Wb, G.ldb(), G.K, G.ldb()};
  L.no_swap = true;
  L.out = dx;
  L.ld_out = G.K;
  return linear(e, L);
}

bool rms(pi05_engine* e, const bf16* x, bf16* y, int ld_y, const bf16* scale, const bf16* shift, int R, int D,
         int rows_per_mod, int mod_ld) {
  return launch(e, rmsnorm_kernel, dim3(rows_grid(R)), dim3(256), 0, false, x, y, scale, shift, R, D, rows_per_mod,
                mod_ld, ld_y);
}
bool rms_bwd(pi05_engine* e, const bf16* x, const bf16* dy, int ld_dy, const bf16* scale, int rows_per_mod,
             int mod_ld, float* gx, int R, int D) {
  const bool vec = ld_dy % 8 == 0 && mod_ld % 8 == 0 && (((uintptr_t)x | (uintptr_t)dy | (uintptr_t)scale) & 15) == 0;
  if (vec && D == 2048)
    return launch(e, rmsnorm_bwd_vec_kernel<8>, dim3(rows_grid(R)), dim3(256), 0, false, x, dy, ld_dy, scale,
                  rows_per_mod, mod_ld, gx, R);
  if (vec && D == 1024)
    return launch(e, rmsnorm_bwd_vec_kernel<4>, dim3(rows_grid(R)), dim3(256), 0, false, x, dy, ld_dy, scale,
                  rows_per_mod, mod_ld, gx, R);
  return launch(e, rmsnorm_bwd_kernel, dim3(rows_grid(R)), dim3(256), 0, false, x, dy, ld_dy, scale, rows_per_mod,
                mod_ld, gx, R, D);
}
// fp32 residual-stream gradient -> bf16 rows of ld_out (times the per-sample gate when given)
bool grad_bf16(pi05_engine* e, const float* g, bf16* out, int ld_out, const bf16* gate, int rows_per_gate, int gate_ld,
               int R, int D) {
  if (D % 8 == 0 && ld_out % 8 == 0 && gate_ld % 8 == 0 && (((uintptr_t)out | (uintptr_t)gate) & 15) == 0) {
    const long n = (long)R * (D / 8);
    return launch(e, grad_to_bf16_vec_kernel, dim3((n + 255) / 256), dim3(256), 0, false, g, out, ld_out, gate,
                  rows_per_gate, gate_ld, R, D);
  }
  const long n = (long)R * D;
  return launch(e, grad_to_bf16_kernel, dim3((n + 255) / 256), dim3(256), 0, false, g, out, ld_out, gate, rows_per_gate,
                gate_ld, R, D);
}

// ------------------------------------------------------------------ forward of one stack-layer
struct StackCtx {
  bool prefix;
  int R, per_sample, pos_off, D, F;
  const bf16* mrow1;  // adaptive norm rows (suffix) or plain scale (prefix)
  const bf16* mrow2;
  int mod_ld;
};

bool fwd_qkv(pi05_engine* e, const LoraGroup& G, const StackCtx& c, Saved& S) {
  if (!rms(e, S.xin, S.h1, c.D + 48, c.mrow1, c.prefix ? nullptr : c.mrow1 + c.D, c.R, c.D, c.per_sample, c.mod_ld))
    return false;
  if (!lora_u(e, G, S.h1, c.R, S.uT_qkv)) return false;
  Lin q{S.h1, G.ldf(), c.R, G.Wf, G.ldf(), P5_QKV, G.ldf()};
  q.no_swap = true;
  q.out = S.qkv;
  q.ld_out = P5_QKV;
  if (!linear(e, q)) return false;
  return launch(e, rope_qkv_kernel, dim3(c.R), dim3(256), 0, false, S.qkv, c.R, c.per_sample, c.pos_off,
                S.qkv + P5_QDIM, S.qkv + P5_QDIM + P5_HD, (const float*)e->d_cos, (const float*)e->d_sin, P5_QKV);
}

bool fwd_after_attn(pi05_engine* e, const TrainLayer& t, const StackCtx& c, Saved& S, bf16* xout, const bf16* gate1,
                    const bf16* gate2, int nb) {
  if (!lora_u(e, t.o, S.o, c.R, S.uT_o)) return false;
  Lin o{S.o, t.o.ldf(), c.R, t.o.Wf, t.o.ldf(), c.D, t.o.ldf()};
  o.no_swap = true;
  o.out = S.xmid;
  o.ld_out = c.D;
  o.res = S.xin;
  o.ld_res = c.D;
  if (c.prefix) {
    o.epi = EPI_RESID;
  } else {
    o.epi = EPI_GATED;
    o.gate = gate1;
    o.ld_gate = c.mod_ld;
    o.gate_div = c.per_sample;
  }
  if (!linear(e, o)) return false;
  if (!rms(e, S.xmid, S.h2, c.D + 32, c.mrow2, c.prefix ? nullptr : c.mrow2 + c.D, c.R, c.D, c.per_sample, c.mod_ld))
    return false;
  if (!lora_u(e, t.gu, S.h2, c.R, S.uT_gu)) return false;
  Lin gu{S.h2, t.gu.ldf(), c.R, t.gu.Wf, t.gu.ldf(), 2 * c.F, t.gu.ldf()};
  gu.no_swap = true;
  gu.epi = EPI_GEGLU;
  gu.out = S.act;
  gu.ld_out = c.F + 16;
  gu.out_t = S.gu;
  gu.ld_out_t = 2 * c.F;
  if (!linear(e, gu)) return false;
  if (!lora_u(e, t.dn, S.act, c.R, S.uT_dn)) return false;
  Lin dn{S.act, t.dn.ldf(), c.R, t.dn.Wf, t.dn.ldf(), c.D, t.dn.ldf()};
  dn.no_swap = true;
  dn.out = xout;
  dn.ld_out = c.D;
  dn.res = S.xmid;
  dn.ld_res = c.D;
  if (c.prefix) {
    dn.epi = EPI_RESID;
  } else {
    dn.epi = EPI_GATED;
    dn.gate = gate2;
    dn.ld_gate = c.mod_ld;
    dn.gate_div = c.per_sample;
  }
  (void)nb;
  return linear(e, dn);
}

// ------------------------------------------------------------------ one micro-batch: forward + backward
bool micro_step(pi05_engine* e, int nb, const float* h_t) {
  Trainer* T = e->tr;
  const int L = e->cfg.gemma_layers, P = e->P, H = e->cfg.horizon, NM = e->NM;
  const int Rp = nb * P, Rs = nb * H, MW = NM * 3 * P5_EXP_W;
  Acts& A = e->A;
  // prefix embeddings (frozen SigLIP + text) into layer 0's input
  if (!run_siglip(e, nb)) return false;
  if (e->cfg.n_text > 0 &&
      !launch(e, embed_text_kernel, dim3(e->cfg.n_text, nb), dim3(256), 0, false, (const int32_t*)A.tokens,
              (const bf16*)e->embed, A.px, e->cfg.n_text, P, e->cfg.n_cameras * P5_SIG_TOK))
    return false;
  CK(cudaMemcpyAsync(T->sp[0].xin, A.px, (size_t)Rp * P5_GEM_W * 2, cudaMemcpyDeviceToDevice, e->stream));
  // time conditioning per sample
  {
    std::vector<float> emb((size_t)nb * P5_EXP_W);
    for (int b = 0; b < nb; ++b) p5_time_embedding(h_t[b], P5_EXP_W, emb.data() + (size_t)b * P5_EXP_W);
    CK(cudaMemcpyAsync(T->d_temb, emb.data(), emb.size() * 4, cudaMemcpyHostToDevice, e->stream));
    CK(cudaStreamSynchronize(e->stream));  // emb lives on the host stack
    const int warps = nb * P5_EXP_W;
    linear_swish_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, e->stream>>>(T->d_temb, e->tin_w, e->tin_b, T->d_c1,
                                                                            (bf16*)nullptr, nb, P5_EXP_W);
    linear_swish_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, e->stream>>>(T->d_c1, e->tout_w, e->tout_b, T->d_c2,
                                                                            T->d_cond, nb, P5_EXP_W);
    CK(cudaGetLastError());
    Lin m{T->d_cond, P5_EXP_W, nb, e->ada_w, P5_EXP_W, MW, P5_EXP_W};
    m.out = T->mods;
    m.ld_out = MW;
    m.bias = e->ada_b;
    if (!linear(e, m)) return false;
  }
  // suffix input
  {
    const long n = (long)Rs * P5_ACT_D;
    flow_inputs_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(T->d_eps, T->d_act, T->d_t, T->d_xt, T->d_u, H, nb);
    if (!launch(e, action_in_kernel, dim3((Rs * P5_EXP_W + 255) / 256), dim3(256), 0, false, (const float*)T->d_xt,
                (const bf16*)e->ain_w, (const bf16*)e->ain_b, T->ss[0].xin, Rs, P5_EXP_W, (float*)nullptr, 0))
      return false;
  }
  // ---------------- forward
  for (int l = 0; l < L; ++l) {
    Saved& Sp = T->sp[l];
    Saved& Ss = T->ss[l];
    const bool last = l == L - 1;
    StackCtx cp{true, Rp, P, 0, P5_GEM_W, P5_GEM_MLP, e->gem[l].rms1, e->gem[l].rms2, 0};
    StackCtx cs{false, Rs, H, P, P5_EXP_W, P5_EXP_MLP, T->mods + (size_t)(2 * l) * 3 * P5_EXP_W,
                T->mods + (size_t)(2 * l + 1) * 3 * P5_EXP_W, MW};
    if (!fwd_qkv(e, T->gl[l].qkv, cp, Sp) || !fwd_qkv(e, T->el[l].qkv, cs, Ss)) return false;
    AttnArgs at = {};
    at.G = P5_NH;
    at.qdiv = 1.0f;
    at.splits = 1;
    if (!last) {  // prefix rows attend the prefix
      at.q = Sp.qkv;
      at.ldq = P5_QKV;
      at.q_bstride = (long)P * P5_QKV;
      at.out = Sp.o;
      at.ldo = P5_QDIM + 16;
      at.o_bstride = (long)P * (P5_QDIM + 16);
      at.k1 = Sp.qkv + P5_QDIM;
      at.v1 = Sp.qkv + P5_QDIM + P5_HD;
      at.ld1 = P5_QKV;
      at.len1 = P;
      at.b1stride = (long)P * P5_QKV;
      at.k2 = at.k1;
      at.v2 = at.v1;
      at.T = P;
      at.lse = Sp.lse;
      at.lse_b = (long)P * P5_NH;
      if (!attention(e, at, nb, P5_HD)) return false;
    }
    // suffix rows attend [prefix || suffix]
    at.q = Ss.qkv;
    at.ldq = P5_QKV;
    at.q_bstride = (long)H * P5_QKV;
    at.out = Ss.o;
    at.ldo = P5_QDIM + 16;
    at.o_bstride = (long)H * (P5_QDIM + 16);
    at.k1 = Sp.qkv + P5_QDIM;
    at.v1 = Sp.qkv + P5_QDIM + P5_HD;
    at.ld1 = P5_QKV;
    at.len1 = P;
    at.b1stride = (long)P * P5_QKV;
    at.k2 = Ss.qkv + P5_QDIM;
    at.v2 = Ss.qkv + P5_QDIM + P5_HD;
    at.ld2 = P5_QKV;
    at.len2 = H;
    at.b2stride = (long)H * P5_QKV;
    at.T = H;
    at.lse = Ss.lse;
    at.lse_b = (long)H * P5_NH;
    if (!attention(e, at, nb, P5_HD)) return false;
    bf16* xo_p = last ? T->xin_p_final : T->sp[l + 1].xin;
    bf16* xo_s = last ? T->xin_s_final : T->ss[l + 1].xin;
    if (!last && !fwd_after_attn(e, T->gl[l], cp, Sp, xo_p, nullptr, nullptr, nb)) return false;
    if (!fwd_after_attn(e, T->el[l], cs, Ss, xo_s, cs.mrow1 + 2 * P5_EXP_W, cs.mrow2 + 2 * P5_EXP_W, nb)) return false;
  }
  // final adaRMS, v, loss
  const bf16* mf = T->mods + (size_t)(NM - 1) * 3 * P5_EXP_W;
  if (!rms(e, T->xin_s_final, T->hf, P5_EXP_W, mf, mf + P5_EXP_W, Rs, P5_EXP_W, H, MW)) return false;
  const float inv_count = 1.0f / ((float)T->n_total * H * P5_ACT_D);
  out_proj_loss_kernel<<<Rs, 1024, 0, e->stream>>>(T->hf, e->aout_w, e->aout_b, T->d_u, T->d_dv, T->d_rowloss, Rs,
                                                   P5_EXP_W, inv_count);
  sum_rows_kernel<<<1, 256, 0, e->stream>>>(T->d_rowloss, Rs, inv_count, T->d_loss);
  // ---------------- backward
  out_proj_bwd_kernel<<<(Rs * P5_EXP_W + 255) / 256, 256, 0, e->stream>>>(T->d_dv, e->aout_w, T->dh_s, Rs, P5_EXP_W);
  CK(cudaMemsetAsync(T->gx_s, 0, (size_t)Rs * P5_EXP_W * 4, e->stream));
  CK(cudaMemsetAsync(T->gx_p, 0, (size_t)Rp * P5_GEM_W * 4, e->stream));
  if (!rms_bwd(e, T->xin_s_final, T->dh_s, P5_EXP_W, mf, H, MW, T->gx_s, Rs, P5_EXP_W)) return false;
  for (int l = L - 1; l >= 0; --l) {
    Saved& Sp = T->sp[l];
    Saved& Ss = T->ss[l];
    const TrainLayer& tp = T->gl[l];
    const TrainLayer& ts = T->el[l];
    const bool last = l == L - 1;
    const bf16* m1 = T->mods + (size_t)(2 * l) * 3 * P5_EXP_W;
    const bf16* m2 = T->mods + (size_t)(2 * l + 1) * 3 * P5_EXP_W;
    // stack-generic MLP + O backward
    auto mlp_o_bwd = [&](bool prefix) -> bool {
      const int R = prefix ? Rp : Rs, D = prefix ? P5_GEM_W : P5_EXP_W, F = prefix ? P5_GEM_MLP : P5_EXP_MLP;
      const TrainLayer& t = prefix ? tp : ts;
      Saved& S = prefix ? Sp : Ss;
      float* gx = prefix ? T->gx_p : T->gx_s;
      bf16* dy = prefix ? T->dy_p : T->dy_s;
      bf16* dact = prefix ? T->dact_p : T->dact_s;
      bf16* dgu = prefix ? T->dgu_p : T->dgu_s;
      bf16* dh = prefix ? T->dh_p : T->dh_s;
      bf16* dO = prefix ? T->do_p : T->do_s;
      const int rpg = prefix ? 1 : H, gld = prefix ? 0 : MW;
      // down projection (gated for the suffix)
      if (!grad_bf16(e, gx, dy, D + 16, prefix ? (const bf16*)nullptr : m2 + 2 * D, rpg, gld, R, D)) return false;
      if (!lora_v(e, t.dn, dy, R, T->vT) || !lora_wgrad(e, T, t.dn, dy, S.act, S.uT_dn, T->vT, R)) return false;
      Lin da{dy, t.dn.ldb(), R, t.dn.Wb, t.dn.ldb(), F, t.dn.ldb()};
      da.no_swap = true;
      if (e->fuse_geglu_bwd) {
        // dact never reaches memory: the epilogue turns each row's 32 dact values into the (dgate, dup) pairs
        da.epi = EPI_GEGLU_BWD;
        da.out = dgu;
        da.ld_out = 2 * F + 32;
        da.res = S.gu;
        da.ld_res = 2 * F;
        if (!linear(e, da)) return false;
      } else {
        da.out = dact;
        da.ld_out = F;
        if (!linear(e, da)) return false;
        static_assert(P5_GEM_MLP % 8 == 0 && P5_EXP_MLP % 8 == 0, "geglu_bwd_kernel takes 8 pairs per thread");
        const long ng = (long)R * (F / 8);
        if (!launch(e, geglu_bwd_kernel, dim3((ng + 255) / 256), dim3(256), 0, false, (const bf16*)S.gu,
                    (const bf16*)dact, F, dgu, 2 * F + 32, R, F))
          return false;
      }
      if (!lora_v(e, t.gu, dgu, R, T->vT) || !lora_wgrad(e, T, t.gu, dgu, S.h2, S.uT_gu, T->vT, R)) return false;
      if (!lora_dx(e, t.gu, dgu, R, dh)) return false;
      if (!rms_bwd(e, S.xmid, dh, D, prefix ? e->gem[l].rms2 : m2, rpg, gld, gx, R, D)) return false;
      // output projection
      if (!grad_bf16(e, gx, dy, D + 16, prefix ? (const bf16*)nullptr : m1 + 2 * D, rpg, gld, R, D)) return false;
      if (!lora_v(e, t.o, dy, R, T->vT) || !lora_wgrad(e, T, t.o, dy, S.o, S.uT_o, T->vT, R)) return false;
      Lin dov{dy, t.o.ldb(), R, t.o.Wb, t.o.ldb(), P5_QDIM, t.o.ldb()};
      dov.no_swap = true;
      dov.out = dO;
      dov.ld_out = P5_QDIM;
      return linear(e, dov);
    };
    if (!mlp_o_bwd(false)) return false;
    if (!last && !mlp_o_bwd(true)) return false;
    // attention backward
    if (!launch(e, attn_dot_kernel, dim3(rows_grid((long)Rs * P5_NH)), dim3(256), 0, false, (const bf16*)T->do_s,
                P5_QDIM, (const bf16*)Ss.o, P5_QDIM + 16, T->Ds, Rs))
      return false;
    if (!last && !launch(e, attn_dot_kernel, dim3(rows_grid((long)Rp * P5_NH)), dim3(256), 0, false,
                         (const bf16*)T->do_p, P5_QDIM, (const bf16*)Sp.o, P5_QDIM + 16, T->Dp, Rp))
      return false;
    QSeg qs_s{Ss.qkv, P5_QKV, (long)H * P5_QKV, T->do_s, P5_QDIM, (long)H * P5_QDIM, Ss.lse, T->Ds, (long)H * P5_NH, H};
    QSeg qs_p{Sp.qkv, P5_QKV, (long)P * P5_QKV, T->do_p, P5_QDIM, (long)P * P5_QDIM, Sp.lse, T->Dp, (long)P * P5_NH, P};
    AttnBwdArgs ab = {};
    ab.k1 = Sp.qkv + P5_QDIM;
    ab.v1 = Sp.qkv + P5_QDIM + P5_HD;
    ab.ld1 = P5_QKV;
    ab.len1 = P;
    ab.b1stride = (long)P * P5_QKV;
    ab.k2 = Ss.qkv + P5_QDIM;
    ab.v2 = Ss.qkv + P5_QDIM + P5_HD;
    ab.ld2 = P5_QKV;
    ab.len2 = H;
    ab.b2stride = (long)H * P5_QKV;
    // dq of the action queries (keys: prefix || suffix)
    ab.qs = qs_s;
    ab.dq = T->dqkv_s;
    ab.ld_dq = P5_QKV + 48;
    ab.dq_b = (long)H * (P5_QKV + 48);
    if (!attn_bwd_dq(e, ab, nb)) return false;
    if (!last) {  // dq of the prefix queries (keys: prefix only)
      AttnBwdArgs ap = ab;
      ap.len2 = 0;
      ap.qs = qs_p;
      ap.dq = T->dqkv_p;
      ap.dq_b = (long)P * (P5_QKV + 48);
      if (!attn_bwd_dq(e, ap, nb)) return false;
    } else {
      CK(cudaMemset2DAsync(T->dqkv_p, (size_t)(P5_QKV + 48) * 2, 0, (size_t)P5_QDIM * 2, Rp, e->stream));
    }
    // dK, dV of the prefix keys: prefix queries (unless last) then action queries
    AttnBwdArgs ak = ab;
    ak.kseg = 1;
    ak.nq = last ? 1 : 2;
    ak.qa = last ? qs_s : qs_p;
    ak.qbseg = qs_s;
    ak.ld_dkv = P5_QKV + 48;
    ak.dkv_b = (long)P * (P5_QKV + 48);
    ak.dk = T->dqkv_p + P5_QDIM;
    ak.dv = T->dqkv_p + P5_QDIM + P5_HD;
    if (!attn_bwd_dkv(e, T, ak, nb)) return false;
    // dK, dV of the suffix keys: action queries only
    AttnBwdArgs as = ab;
    as.kseg = 2;
    as.nq = 1;
    as.qa = qs_s;
    as.ld_dkv = P5_QKV + 48;
    as.dkv_b = (long)H * (P5_QKV + 48);
    as.dk = T->dqkv_s + P5_QDIM;
    as.dv = T->dqkv_s + P5_QDIM + P5_HD;
    if (!attn_bwd_dkv(e, T, as, nb)) return false;
    // RoPE backward, then the q/k/v projections of both stacks
    if (!launch(e, rope_bwd_kernel, dim3(Rs), dim3(256), 0, false, T->dqkv_s, P5_QKV + 48, Rs, H, P,
                (const float*)e->d_cos, (const float*)e->d_sin, 1) ||
        !launch(e, rope_bwd_kernel, dim3(Rp), dim3(256), 0, false, T->dqkv_p, P5_QKV + 48, Rp, P, 0,
                (const float*)e->d_cos, (const float*)e->d_sin, last ? 0 : 1))
      return false;
    auto qkv_bwd = [&](bool prefix) -> bool {
      const int R = prefix ? Rp : Rs, D = prefix ? P5_GEM_W : P5_EXP_W;
      const LoraGroup& G = prefix ? tp.qkv : ts.qkv;
      Saved& S = prefix ? Sp : Ss;
      bf16* dq = prefix ? T->dqkv_p : T->dqkv_s;
      bf16* dh = prefix ? T->dh_p : T->dh_s;
      if (!lora_v(e, G, dq, R, T->vT) || !lora_wgrad(e, T, G, dq, S.h1, S.uT_qkv, T->vT, R)) return false;
      if (!lora_dx(e, G, dq, R, dh)) return false;
      return rms_bwd(e, S.xin, dh, D, prefix ? e->gem[l].rms1 : m1, prefix ? 1 : H, prefix ? 0 : MW,
                     prefix ? T->gx_p : T->gx_s, R, D);
    };
    if (!qkv_bwd(false) || !qkv_bwd(true)) return false;
    if (T->overlap) {  // layer l's adapter gradients (both stacks) are final: average them over the ranks
      CK(cudaEventRecord(T->dp->layer_done[l], e->stream));
      for (const TrainLayer* tl : {&tp, &ts}) {
        const long a = tl->qkv.offA[0], b = tl->dn.offB[0] + 16L * tl->dn.Fa[0];
        if (!dp_average(e, T->dp, T->g + a, (size_t)(b - a), T->dp->layer_done[l])) return false;
      }
    }
  }
  if (T->overlap && !dp_average(e, T->dp, T->d_loss, 1, nullptr)) return false;
  return true;
}

bool lora_accumulate(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* actions,
                     const float* noise, const float* t, bool exchange = false) {
  Trainer* T = e->tr;
  const int H = e->cfg.horizon;
  const size_t ib = (size_t)e->cfg.n_cameras * P5_IMG * P5_IMG * 3;
  // the gradient buffer and the loss hold the mean over every sample accumulated since the last zero:
  // re-weight what is there by c / (c + n), and let this call's samples add with weight 1 / (c + n)
  const int c = T->n_seen;
  if (c > 0) {
    const float w = (float)c / (float)(c + n);
    scale_f32_kernel<<<148 * 4, 256, 0, e->stream>>>(T->g, T->n_params, w);
    scale_f32_kernel<<<1, 32, 0, e->stream>>>(T->d_loss, 1, w);
    CK(cudaGetLastError());
  }
  T->n_total = c + n;
  T->n_seen = c + n;
  for (int b0 = 0; b0 < n; b0 += T->mb) {
    const int nb = std::min(T->mb, n - b0);
    CK(cudaMemcpyAsync(e->A.images, images + b0 * ib, nb * ib, cudaMemcpyDefault, e->stream));
    if (e->cfg.n_text > 0)
      CK(cudaMemcpyAsync(e->A.tokens, tokens + (size_t)b0 * e->cfg.n_text, (size_t)nb * e->cfg.n_text * 4,
                         cudaMemcpyDefault, e->stream));
    const size_t ab = (size_t)H * P5_ACT_D * 4;
    CK(cudaMemcpyAsync(T->d_act, actions + (size_t)b0 * H * P5_ACT_D, nb * ab, cudaMemcpyDefault, e->stream));
    CK(cudaMemcpyAsync(T->d_eps, noise + (size_t)b0 * H * P5_ACT_D, nb * ab, cudaMemcpyDefault, e->stream));
    std::vector<float> th(nb);
    CK(cudaMemcpy(th.data(), t + b0, nb * 4, cudaMemcpyDefault));
    CK(cudaMemcpyAsync(T->d_t, th.data(), nb * 4, cudaMemcpyHostToDevice, e->stream));
    // with `exchange`, the last micro-batch averages each finished layer over the ranks during its backward
    T->overlap = exchange && T->dp && b0 + nb >= n;
    const bool ok = micro_step(e, nb, th.data());
    T->overlap = false;
    if (!ok) return false;
  }
  T->reduced = exchange && T->dp;
  return true;
}

// Gradients and loss averaged over the ranks (when attached) before the optimizer reads them.
bool lora_exchange(pi05_engine* e) {
  Trainer* T = e->tr;
  if (!T->dp) return true;
  if (!T->reduced && (!dp_average(e, T->dp, T->g, (size_t)T->n_params, nullptr) ||
                      !dp_average(e, T->dp, T->d_loss, 1, nullptr)))
    return false;
  T->reduced = false;
  return dp_join(e, T->dp);
}

// openpi's warmup + cosine schedule (optax warmup_cosine_decay_schedule with init lr / (warmup + 1)), in
// double precision and rounded once, as the host computes it before each update
float lora_schedule_lr(const pi05_lora_config& c, int k) {
  if (c.warmup_steps <= 0 && c.decay_steps <= 0) return c.lr;
  const double peak = c.lr, end = c.decay_lr, w = c.warmup_steps;
  if (k < c.warmup_steps) {
    const double init = peak / (w + 1.0);
    return (float)(init + (peak - init) * (double)k / w);
  }
  const double span = std::max(1.0, (double)c.decay_steps - w);
  const double t = std::min((double)k - w, span);
  return (float)(end + (peak - end) * 0.5 * (1.0 + std::cos(M_PI * t / span)));
}

bool lora_opt(pi05_engine* e) {
  Trainer* T = e->tr;
  const int nb = 256;
  sumsq_partial_kernel<<<nb, 256, 0, e->stream>>>(T->g, T->n_params, T->sumsq);
  const float lr = lora_schedule_lr(T->cfg, T->step);  // update number T->step (0-based) of the schedule
  T->step += 1;
  adamw_kernel<<<148 * 8, 256, 0, e->stream>>>(T->p, T->g, T->m, T->v, T->n_params, T->sumsq, nb, T->cfg.clip_norm,
                                               lr, T->cfg.beta1, T->cfg.beta2, T->cfg.eps, T->cfg.weight_decay,
                                               T->step);
  if (T->ema) ema_kernel<<<148 * 4, 256, 0, e->stream>>>(T->ema, T->p, T->n_params, T->cfg.ema_decay);
  CK(cudaGetLastError());
  return scatter_all(e, T);
}

}  // namespace

// ===================================================================== C ABI (LoRA)
extern "C" {

void pi05_lora_default_config(pi05_lora_config* c) {
  if (!c) return;
  c->rank = 16;
  c->alpha = 32.0f;
  c->lr = 1e-4f;
  c->beta1 = 0.9f;
  c->beta2 = 0.95f;
  c->eps = 1e-8f;
  c->weight_decay = 1e-10f;
  c->clip_norm = 1.0f;
  c->micro_batch = 8;
  c->warmup_steps = 0;
  c->decay_steps = 0;
  c->decay_lr = 0.f;
  c->ema_decay = 0.f;
}

float pi05_lora_schedule_lr(const pi05_lora_config* c, int k) { return c ? lora_schedule_lr(*c, k) : 0.f; }

int pi05_lora_get_ema(pi05_engine* e, float* out) {
  if (!e || !e->tr || !e->tr->ema) return PI05_ERR_STATE;
  if (!out) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  if (cudaMemcpy(out, e->tr->ema, e->tr->n_params * 4, cudaMemcpyDefault) != cudaSuccess) return PI05_ERR_CUDA;
  return PI05_OK;
}

int pi05_lora_init(pi05_engine* e, const pi05_lora_config* c, uint64_t seed) {
  if (!e || !e->weights_ready) return PI05_ERR_STATE;
  pi05_lora_config cfg;
  pi05_lora_default_config(&cfg);
  if (c) cfg = *c;
  if (e->cfg.text_pad_mask || e->cfg.prefix_group) {
    e->err = "pi05_lora_init: the LoRA step trains on full prompts with one prefix attention group "
             "(text_pad_mask and prefix_group must be 0)";
    return PI05_ERR_ARG;
  }
  if (e->kv_mix) {
    e->err = "pi05_lora_init: the LoRA step trains without KV layer mixing (pi05_set_kv_mix NULL first)";
    return PI05_ERR_STATE;
  }
  if (cfg.rank != 16 || cfg.alpha != 32.0f || cfg.micro_batch < 1) {
    e->err = "pi05_lora_init: this build implements rank 16, alpha 32";
    return PI05_ERR_ARG;
  }
  if (e->tr) {
    e->err = "pi05_lora_init: already initialised";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  if (!lora_create(e, &cfg, seed)) return fail_code(e);
  return PI05_OK;
}

long pi05_lora_num_params(pi05_engine* e) { return (e && e->tr) ? e->tr->n_params : -1; }

int pi05_lora_zero_grads(pi05_engine* e) {
  if (!e || !e->tr) return PI05_ERR_STATE;
  cudaSetDevice(e->device);
  if (cudaMemsetAsync(e->tr->g, 0, e->tr->n_params * 4, e->stream) != cudaSuccess ||
      cudaMemsetAsync(e->tr->d_loss, 0, 4, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  e->tr->n_seen = 0;
  return PI05_OK;
}

int pi05_lora_accumulate(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* actions,
                         const float* noise, const float* t, float* loss) {
  if (!e || !e->tr) return PI05_ERR_STATE;
  if (n < 1 || !images || !actions || !noise || !t || (e->cfg.n_text > 0 && !tokens)) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  if (!lora_accumulate(e, n, images, tokens, actions, noise, t)) return fail_code(e);
  if (loss) {
    if (cudaMemcpyAsync(loss, e->tr->d_loss, 4, cudaMemcpyDefault, e->stream) != cudaSuccess) return PI05_ERR_CUDA;
    return pi05_sync(e);
  }
  return PI05_OK;
}

int pi05_lora_opt_step(pi05_engine* e) {
  if (!e || !e->tr) return PI05_ERR_STATE;
  cudaSetDevice(e->device);
  if (!lora_exchange(e) || !lora_opt(e)) return fail_code(e);
  return PI05_OK;
}

int pi05_lora_step(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* actions,
                   const float* noise, const float* t, float* loss) {
  int rc = pi05_lora_zero_grads(e);
  if (rc != PI05_OK) return rc;
  if (n < 1 || !images || !actions || !noise || !t || (e->cfg.n_text > 0 && !tokens)) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  // one accumulate pass whose backward averages each finished layer over the ranks (data parallelism)
  if (!lora_accumulate(e, n, images, tokens, actions, noise, t, true)) return fail_code(e);
  rc = pi05_lora_opt_step(e);
  if (rc != PI05_OK) return rc;
  if (loss) {
    if (cudaMemcpyAsync(loss, e->tr->d_loss, 4, cudaMemcpyDefault, e->stream) != cudaSuccess) return PI05_ERR_CUDA;
    return pi05_sync(e);
  }
  return PI05_OK;
}

static int lora_copy(pi05_engine* e, float* dst, const float* src) {
  if (!e || !e->tr || !dst) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  if (cudaMemcpyAsync(dst, src, e->tr->n_params * 4, cudaMemcpyDefault, e->stream) != cudaSuccess) return PI05_ERR_CUDA;
  return pi05_sync(e);
}
int pi05_lora_get_params(pi05_engine* e, float* out) { return e && e->tr ? lora_copy(e, out, e->tr->p) : PI05_ERR_STATE; }
int pi05_lora_get_grads(pi05_engine* e, float* out) { return e && e->tr ? lora_copy(e, out, e->tr->g) : PI05_ERR_STATE; }
int pi05_lora_set_params(pi05_engine* e, const float* in) {
  if (!e || !e->tr || !in) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  if (cudaMemcpyAsync(e->tr->p, in, e->tr->n_params * 4, cudaMemcpyDefault, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  // new adapters: the EMA restarts from them
  if (e->tr->ema && cudaMemcpyAsync(e->tr->ema, e->tr->p, e->tr->n_params * 4, cudaMemcpyDeviceToDevice,
                                    e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  if (!scatter_all(e, e->tr)) return fail_code(e);
  return pi05_sync(e);
}
void* pi05_lora_grad_buffer(pi05_engine* e) { return e && e->tr ? (void*)e->tr->g : nullptr; }

int pi05_lora_reset_optimizer(pi05_engine* e) {
  if (!e || !e->tr) return PI05_ERR_STATE;
  cudaSetDevice(e->device);
  Trainer* T = e->tr;
  if (cudaMemsetAsync(T->m, 0, T->n_params * 4, e->stream) != cudaSuccess ||
      cudaMemsetAsync(T->v, 0, T->n_params * 4, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  T->step = 0;
  return pi05_sync(e);
}

// Train state file: "pi05lora 1\nparams N\nstep S\nema E\n" padded to 256 bytes, then p, m, v (fp32, N each)
// and, when E = 1, the EMA.
int pi05_lora_save_state(pi05_engine* e, const char* path) {
  if (!e || !e->tr || !path) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  Trainer* T = e->tr;
  std::vector<float> buf((size_t)T->n_params);
  FILE* f = fopen(path, "wb");
  if (!f) {
    e->err = std::string("cannot open ") + path;
    return PI05_ERR_ARG;
  }
  char hdr[256] = {0};
  snprintf(hdr, sizeof(hdr), "pi05lora 1\nparams %ld\nstep %d\nema %d\n", T->n_params, T->step, T->ema ? 1 : 0);
  fwrite(hdr, 1, sizeof(hdr), f);
  for (float* src : {T->p, T->m, T->v, T->ema}) {
    if (!src) continue;
    if (cudaMemcpy(buf.data(), src, T->n_params * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
      fclose(f);
      return PI05_ERR_CUDA;
    }
    fwrite(buf.data(), 4, buf.size(), f);
  }
  fclose(f);
  return PI05_OK;
}

int pi05_lora_load_state(pi05_engine* e, const char* path) {
  if (!e || !e->tr || !path) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  Trainer* T = e->tr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    e->err = std::string("cannot open ") + path;
    return PI05_ERR_ARG;
  }
  char hdr[256];
  long np = -1;
  int step = -1;
  int ema = 0;
  if (fread(hdr, 1, sizeof(hdr), f) != sizeof(hdr) ||
      sscanf(hdr, "pi05lora 1\nparams %ld\nstep %d\nema %d", &np, &step, &ema) < 2 || np != T->n_params ||
      (ema != 0) != (T->ema != nullptr)) {
    fclose(f);
    e->err = "pi05_lora_load_state: not a train state of this configuration";
    return PI05_ERR_ARG;
  }
  std::vector<float> buf((size_t)np);
  for (float* dst : {T->p, T->m, T->v, T->ema}) {
    if (!dst) continue;
    if (fread(buf.data(), 4, buf.size(), f) != buf.size()) {
      fclose(f);
      e->err = "pi05_lora_load_state: short file";
      return PI05_ERR_ARG;
    }
    if (cudaMemcpy(dst, buf.data(), np * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      fclose(f);
      return PI05_ERR_CUDA;
    }
  }
  fclose(f);
  T->step = step;
  if (!scatter_all(e, T)) return fail_code(e);
  return pi05_sync(e);
}


int pi05_nccl_unique_id(void* id) {
  if (!id) return PI05_ERR_ARG;
  NcclApi& A = nccl_api();
  if (!A.ok) return PI05_ERR_STATE;
  ncclUniqueId u;
  if (A.get_unique_id(&u) != ncclSuccess) return PI05_ERR_CUDA;
  memcpy(id, &u, sizeof(u));
  return PI05_OK;
}

int pi05_lora_attach_nccl(pi05_engine* e, const void* id, int rank, int world) {
  if (!e) return PI05_ERR_ARG;
  if (!e->tr) {
    e->err = "pi05_lora_attach_nccl: call pi05_lora_init first";
    return PI05_ERR_STATE;
  }
  if (!id || world < 1 || rank < 0 || rank >= world) {
    e->err = "pi05_lora_attach_nccl: needs 0 <= rank < world and the 128-byte unique id";
    return PI05_ERR_ARG;
  }
  if (e->tr->dp) {
    e->err = "pi05_lora_attach_nccl: already attached";
    return PI05_ERR_STATE;
  }
  NcclApi& A = nccl_api();
  if (!A.ok) {
    e->err = "pi05_lora_attach_nccl: " + A.why;
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  DpComm* d = new DpComm();
  d->rank = rank;
  d->world = world;
  auto fail = [&](int code) {
    if (d->comm) A.comm_abort(d->comm);
    d->comm = nullptr;
    dp_release(d);
    return code;
  };
  if (cudaStreamCreateWithFlags(&d->cs, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&d->reduced, cudaEventDisableTiming) != cudaSuccess)
    return fail(PI05_ERR_CUDA);
  d->layer_done.assign(e->cfg.gemma_layers, nullptr);
  for (cudaEvent_t& ev : d->layer_done)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return fail(PI05_ERR_CUDA);
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // init and collectives return at once; every wait on them is bounded (nccl_settle)
  const ncclResult_t r = A.init_rank_config(&d->comm, world, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    e->err = std::string("ncclCommInitRankConfig: ") + A.error_string(r);
    return fail(PI05_ERR_CUDA);
  }
  if (!nccl_settle(e, d->comm, "ncclCommInitRankConfig")) return fail(PI05_ERR_CUDA);
  e->tr->dp = d;
  return PI05_OK;
}

int pi05_lora_world(pi05_engine* e) { return (e && e->tr && e->tr->dp) ? e->tr->dp->world : 1; }

}  // extern "C"

// engine.cu — host side of the pi0.5 engine: weight arena, activation buffers, launch planning,
// CUDA-graph capture, and the C ABI declared in include/pi05.h.
//
// Reference boundary replaced: include/pi05_batch.h of the deleted engine
// (docs/archive/windows/π05_네이티브엔진.md:288-303).  The reference captured the per-board prefix as
// one CUDA graph and ran the denoise for all boards at once (:298); here both the prefill and the
// 10-step denoise of a batch are captured once per batch size and replayed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/pi05.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "attention_sig.cuh"
#include "gemm_wide.cuh"
#include "gemm_pair.cuh"
#include "denoise_mega.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "resize.cuh"

using namespace p5;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Tensor {
  std::string name;
  bf16* ptr;
  long rows;
  int cols;
};

struct SigLayer {
  bf16 *ln1s, *ln1b, *wqkv, *bqkv, *wo, *bo, *ln2s, *ln2b, *w1, *b1, *w2, *b2;
};
struct GemLayer {
  bf16 *rms1, *wqkv, *wo, *rms2, *wgu, *wd;
};
struct ExpLayer {
  bf16 *wqkv, *wo, *wgu, *wd;
};

struct Acts {
  uint8_t* images;
  int32_t* tokens;
  bf16 *patches, *sx, *sy, *sqkv, *so, *sh;
  bf16 *px, *ph, *pqkv, *po, *pact, *kcache, *vcache;
  bf16 *ex, *eh, *eqkv, *eo, *eact, *ek, *ev;
  float *xt, *noise, *actions;
};

}  // namespace

struct pi05_engine {
  pi05_config cfg;
  int device = 0, max_batch = 1, P = 968, NM = 37;
  cudaStream_t stream = nullptr;
  std::string err;
  int* d_status = nullptr;
  EncodeTiledFn encode = nullptr;
  int num_sms = 148;
  bool pdl = true;

  std::vector<void*> allocs;
  char* warena = nullptr;
  size_t wbytes = 0, wused = 0;
  std::vector<Tensor> tensors;

  // weights
  bf16 *sig_stem_w, *sig_stem_b, *sig_posemb, *sig_post_s, *sig_post_b, *sig_head_w, *sig_head_b;
  std::vector<SigLayer> sig;
  bf16* embed;
  std::vector<GemLayer> gem;
  std::vector<ExpLayer> ex;
  bf16 *ada_w, *ada_b, *ain_w, *ain_b, *aout_w, *aout_b, *tin_w, *tin_b, *tout_w, *tout_b;

  Acts A;
  float *d_cos = nullptr, *d_sin = nullptr;
  bf16* mods = nullptr;  // [steps][NM*3*1024]
  float* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  int* counters = nullptr;
  int n_counters = 0;
  float *attn_ws_o = nullptr, *attn_ws_ml = nullptr;
  size_t attn_ws_rows = 0;

  bool weights_ready = false;
  int wgen = 0;  // bumped whenever the weights change
  // persistent one-sample denoise (denoise_mega.cuh), opt-in with PI05_MEGA=1: it matches the
  // per-kernel CUDA-graph path (~12 ms per 10-step chunk) but does not beat it yet
  bool mega = false;
  // q/k/v weights with interleaved head rows (fused-RoPE projections), rebuilt when stale
  int qkv_il_wgen = -1;
  bf16* exp_wqkv_il = nullptr;
  bf16* gem_wqkv_il = nullptr;
  CUtensorMap* mega_maps = nullptr;
  unsigned* mega_ctr = nullptr;
  int prefix_n = 0;  // batch whose prefix cache is valid
  std::map<int, cudaGraphExec_t> denoise_graphs, prefill_graphs;
  std::map<int, long> denoise_launches, prefill_launches;
  // pi05_prefill_embeds: the text part of the prefix from the caller's embeddings [max_batch][n_text][2048]
  // instead of token ids, with its own prefill graphs
  bf16* text_emb = nullptr;
  bool text_from_emb = false;
  std::map<int, cudaGraphExec_t> prefill_emb_graphs;
  std::map<int, long> prefill_emb_launches;
  long launches = 0;  // kernels enqueued (counted at capture time)
  struct Trainer* tr = nullptr;  // LoRA train state (train.cuh), created by pi05_lora_init
  bool cluster_splitk = true;    // few-token split-K GEMMs reduce inside a cluster (PI05_CLUSTER_SPLITK=0: tickets)
  bool gemm_wide = true;          // 256x256 tiles for large GEMMs (PI05_GEMM_WIDE=0: 128x256)
  bool gemm_pair = true;          // CTA-pair 256x256 tiles (cta_group::2) for K < 4096 (PI05_GEMM_PAIR=0: one SM)
  int pair_clusters = 0;          // CTA pairs of gemm_pair_kernel that fit on the GPU at once
  bool wide_swap = true;          // few M-tiles: weights-on-M cluster split-K (PI05_WIDE_SWAP=0: normal tiles)
  bool attn_tc = true;           // head_dim-256 MQA attention on tcgen05 (PI05_ATTN_TC=0: the mma.sync kernel)
  bool attn_bwd_pipe = true;     // dQ backward with dS overlapped (PI05_ATTN_BWD_PIPE=0: the one-slot kernel)
  // split-KV partials of the tensor-core attention as fp16 O / l, half the bytes of fp32 O
  // (PI05_ATTN_WS_HALF=0: fp32)
  bool attn_ws_half = true;
  // few-token denoise: adaRMSNorm folded into the q/k/v and gate/up cluster GEMMs, fed by per-token
  // sum-of-squares partials from the producers of x (PI05_FUSE_NORM=0: separate rmsnorm launches)
  bool fuse_norm = true;
  bool fuse_geglu_bwd = true;  // LoRA: GeGLU backward in the down projection's dX epilogue (PI05_FUSE_GEGLU_BWD=0: separate)
  // receding-horizon stepping (pi05_act_batch): per slot the last post-processed chunk [horizon][act_dim],
  // the next row to execute and the plans made (offset of the slot's noise stream)
  int act_dim = P5_ACT_D, act_replan = 16;
  std::vector<float> act_mean, act_std;
  std::vector<uint8_t> act_delta;
  uint64_t act_seed = 0;
  std::vector<std::vector<float>> act_chunk;
  std::vector<int> act_next;
  std::vector<long> act_plans;
  float* noise_chol = nullptr;  // [horizon*32][horizon*32] lower-triangular factor of the noise covariance
  // soft inpainting (pi05_set_inpaint): the first inp_fixed action rows are held to known values after
  // the steps that start above inp_tmin; inp_corr [U][K] = Sigma_UO Sigma_OO^-1, inp_known
  // [max_batch][K], inp_on [max_batch] (0 = that batch position denoises freely), inp_eps the step-0
  // noise of the batch (K = inp_fixed * 32, U = horizon * 32 - K)
  int inp_fixed = 0;
  float inp_tmin = 0.f;
  float *inp_corr = nullptr, *inp_known = nullptr, *inp_eps = nullptr;
  int* inp_on = nullptr;
  // KV layer mixing (pi05_set_kv_mix): the expert's layer l attends to a linear combination of the prefix
  // layers' K (and V); mix_w [2][L][L] and mix_b [2][L][256] (K then V, bf16 values in fp32), the mixed
  // caches laid out as the prefix cache
  bool kv_mix = false;
  float *mix_w = nullptr, *mix_b = nullptr;
  bf16 *kmix = nullptr, *vmix = nullptr;
  // device staging of pi05_act_batch's camera frames: host frames, resize tap tables, frame jobs
  uint8_t* frame_stage = nullptr;
  size_t frame_stage_bytes = 0;
  int32_t* rs_tab = nullptr;
  size_t rs_tab_bytes = 0;
  p5rs::FrameJob* rs_jobs = nullptr;
  size_t rs_jobs_bytes = 0;
  float* nrm_ss = nullptr;  // 2 buffers of [P5_EXP_W / 16 parts][64 tokens]
  // verify run (pi05_verify): named intermediate points of sample 0 are copied to the host and passed
  // to probe_fn after the kernels that produce them; null outside a verify run (and during capture)
  pi05_probe_fn probe_fn = nullptr;
  pi05_plant_fn plant_fn = nullptr;  // teacher-forced verify run: the callback may overwrite the point
  void* probe_ctx = nullptr;
  // prompt padding mask (cfg.text_pad_mask): per batch position, the number of prefix tokens before the
  // prompt's trailing padding (ids 0) -- the keys attended to, and the first position of the action tokens
  int* d_valid = nullptr;
  // single-sample passes at batch position s0 (batch-invariant mode): the bodies offset the per-sample
  // inputs, KV cache and flow state by s0 and share the scratch activations of position 0
  int s0 = 0;
};

namespace {

bool set_err(pi05_engine* e, const std::string& s) {
  e->err = s;
  return false;
}
#define CK(call)                                                                              \
  do {                                                                                        \
    cudaError_t _e = (call);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      set_err(e, std::string(#call) + ": " + cudaGetErrorString(_e) + " @" + std::to_string(__LINE__)); \
      return false;                                                                           \
    }                                                                                         \
  } while (0)

bool dalloc(pi05_engine* e, void** p, size_t bytes) {
  CK(cudaMalloc(p, bytes));
  CK(cudaMemsetAsync(*p, 0, bytes, e->stream));
  e->allocs.push_back(*p);
  return true;
}

bf16* wtake(pi05_engine* e, const std::string& name, long rows, int cols) {
  const size_t bytes = ((size_t)rows * cols * 2 + 255) & ~(size_t)255;
  if (e->warena && e->wused + bytes > e->wbytes) return nullptr;
  bf16* p = e->warena ? reinterpret_cast<bf16*>(e->warena + e->wused) : nullptr;
  e->wused += bytes;
  if (e->warena) e->tensors.push_back({name, p, rows, cols});
  return p;
}

// Lay out every weight tensor (called twice: once to size the arena, once to assign pointers).
void layout_weights(pi05_engine* e) {
  const pi05_config& c = e->cfg;
  e->wused = 0;
  e->tensors.clear();
  e->sig_stem_w = wtake(e, "sig.stem.w", P5_SIG_W, P5_SIG_KPAD);
  e->sig_stem_b = wtake(e, "sig.stem.b", 1, P5_SIG_W);
  e->sig_posemb = wtake(e, "sig.posemb", 256, P5_SIG_W);
  e->sig.resize(c.siglip_layers);
  for (int l = 0; l < c.siglip_layers; ++l) {
    SigLayer& s = e->sig[l];
    const std::string p = "sig.l" + std::to_string(l) + ".";
    s.ln1s = wtake(e, p + "ln1.s", 1, P5_SIG_W);
    s.ln1b = wtake(e, p + "ln1.b", 1, P5_SIG_W);
    s.wqkv = wtake(e, p + "qkv.w", P5_SIG_QKV, P5_SIG_W);
    s.bqkv = wtake(e, p + "qkv.b", 1, P5_SIG_QKV);
    s.wo = wtake(e, p + "o.w", P5_SIG_W, P5_SIG_W);
    s.bo = wtake(e, p + "o.b", 1, P5_SIG_W);
    s.ln2s = wtake(e, p + "ln2.s", 1, P5_SIG_W);
    s.ln2b = wtake(e, p + "ln2.b", 1, P5_SIG_W);
    s.w1 = wtake(e, p + "mlp1.w", P5_SIG_MLP, P5_SIG_W);
    s.b1 = wtake(e, p + "mlp1.b", 1, P5_SIG_MLP);
    s.w2 = wtake(e, p + "mlp2.w", P5_SIG_W, P5_SIG_MLP);
    s.b2 = wtake(e, p + "mlp2.b", 1, P5_SIG_W);
  }
  e->sig_post_s = wtake(e, "sig.post.s", 1, P5_SIG_W);
  e->sig_post_b = wtake(e, "sig.post.b", 1, P5_SIG_W);
  e->sig_head_w = wtake(e, "sig.head.w", P5_GEM_W, P5_SIG_W);
  e->sig_head_b = wtake(e, "sig.head.b", 1, P5_GEM_W);
  e->embed = wtake(e, "gem.embed", P5_VOCAB, P5_GEM_W);
  e->gem.resize(c.gemma_layers);
  for (int l = 0; l < c.gemma_layers; ++l) {
    GemLayer& g = e->gem[l];
    const std::string p = "gem.l" + std::to_string(l) + ".";
    g.rms1 = wtake(e, p + "rms1", 1, P5_GEM_W);
    g.wqkv = wtake(e, p + "qkv.w", P5_QKV, P5_GEM_W);
    g.wo = wtake(e, p + "o.w", P5_GEM_W, P5_QDIM);
    g.rms2 = wtake(e, p + "rms2", 1, P5_GEM_W);
    g.wgu = wtake(e, p + "gu.w", 2 * P5_GEM_MLP, P5_GEM_W);
    g.wd = wtake(e, p + "down.w", P5_GEM_W, P5_GEM_MLP);
  }
  e->ex.resize(c.expert_layers);
  for (int l = 0; l < c.expert_layers; ++l) {
    ExpLayer& x = e->ex[l];
    const std::string p = "exp.l" + std::to_string(l) + ".";
    x.wqkv = wtake(e, p + "qkv.w", P5_QKV, P5_EXP_W);
    x.wo = wtake(e, p + "o.w", P5_EXP_W, P5_QDIM);
    x.wgu = wtake(e, p + "gu.w", 2 * P5_EXP_MLP, P5_EXP_W);
    x.wd = wtake(e, p + "down.w", P5_EXP_W, P5_EXP_MLP);
  }
  e->ada_w = wtake(e, "exp.ada.w", (long)e->NM * 3 * P5_EXP_W, P5_EXP_W);
  e->ada_b = wtake(e, "exp.ada.b", 1, e->NM * 3 * P5_EXP_W);
  e->ain_w = wtake(e, "action_in.w", P5_EXP_W, P5_ACT_D);
  e->ain_b = wtake(e, "action_in.b", 1, P5_EXP_W);
  e->aout_w = wtake(e, "action_out.w", P5_ACT_D, P5_EXP_W);
  e->aout_b = wtake(e, "action_out.b", 1, P5_ACT_D);
  e->tin_w = wtake(e, "time_in.w", P5_EXP_W, P5_EXP_W);
  e->tin_b = wtake(e, "time_in.b", 1, P5_EXP_W);
  e->tout_w = wtake(e, "time_out.w", P5_EXP_W, P5_EXP_W);
  e->tout_b = wtake(e, "time_out.b", 1, P5_EXP_W);
}

// ------------------------------------------------------------------ launch helpers
template <typename... KArgs, typename... Args>
bool launch(pi05_engine* e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, bool pdl, Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = e->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = (pdl && e->pdl) ? 1 : 0;
  lc.attrs = at;
  lc.numAttrs = 1;
  CK(cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...));
  e->launches++;
  return true;
}

bool make_tmap(pi05_engine* e, CUtensorMap* m, const bf16* base, long rows, int K, int ld, int box_rows) {
  if (((uintptr_t)base & 15) || (ld * 2) % 16) return set_err(e, "tensor map: misaligned operand");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = e->encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_err(e, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return true;
}

// general 2-D map: `inner` contiguous elements per row, `rows` rows of stride `ld`, box inner x box_rows
bool make_tmap_box(pi05_engine* e, CUtensorMap* m, const bf16* base, long rows, long inner, int ld, int box_inner,
                   int box_rows) {
  if (((uintptr_t)base & 15) || (ld * 2) % 16) return set_err(e, "tensor map: misaligned operand");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = e->encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_err(e, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return true;
}

// rank-3/4 map with 128-byte swizzle: dims[0] contiguous, strides in bytes for dims 1.., box per dim
bool make_tmap_nd(pi05_engine* e, CUtensorMap* m, const bf16* base, int rank, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box) {
  if ((uintptr_t)base & 15) return set_err(e, "tensor map: misaligned operand");
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) {
      if (strides[i] % 16) return set_err(e, "tensor map: misaligned stride");
      st[i] = strides[i];
    }
  }
  CUresult r = e->encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<bf16*>(base), d, st, bx, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_err(e, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return true;
}

// One linear layer y = x W^T with a fused epilogue.  x: [T][K] (ld ldx), W: [F][K] (ld ldw).
struct Lin {
  const bf16* x;
  int ldx, T;
  const bf16* w;
  int ldw, F, K;
  int epi = EPI_STORE;
  bf16* out = nullptr;
  int ld_out = 0;
  float* out_f32 = nullptr;
  int ld_out_f32 = 0;
  const bf16* bias = nullptr;
  const bf16* res = nullptr;
  int ld_res = 0;
  const bf16* gate = nullptr;
  int ld_gate = 0, gate_div = 1;
  float out_scale = 1.0f;
  const bf16* addend = nullptr;
  int add_ld = 0, add_mod = 1;
  // LoRA path
  bool no_swap = false;  // keep tokens on the 128-row side even for few tokens
  bool amn = false;      // x is [K rows][T columns] read MN-major: D[T][F] = x^T . w^T (weight gradients)
  bf16* out_t = nullptr;
  int ld_out_t = 0;
  int lg_mode = 0, lg_trans = 0, lg_K = 0;
  long lg_off[3] = {0, 0, 0};
  // EPI_ROPE (few-token q/k/v projection with interleaved head rows; see GemmArgs rope_*)
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_pos_off = 0, rope_per_sample = 1, rope_ld_kv = 0;
  const int* rope_base = nullptr;
  bf16* rope_k = nullptr;
  bf16* rope_v = nullptr;
  // fused adaRMSNorm of x (few-token cluster path; see GemmArgs nrm_*) and sum-of-squares partials out
  const float* nrm_ss = nullptr;
  int nrm_ss_ld = 0, nrm_parts = 0, nrm_D = 0;
  const bf16* nrm_scale = nullptr;
  const bf16* nrm_shift = nullptr;
  float* ss_out = nullptr;
  int ss_ld = 0;
};

bool launch_gemm_wide(pi05_engine* e, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga) {
  const dim3 grid(std::min(ga.tiles_m * ga.tiles_n, e->num_sms));
  const size_t sm = (size_t)GemmWideCfg::SMEM;
  const bool p = ga.pdl != 0;
  switch (ga.epi) {
    case EPI_GELU: return launch(e, gemm_wide_kernel<EPI_GELU>, grid, dim3(384), sm, p, ta, tb, ga);
    case EPI_RESID: return launch(e, gemm_wide_kernel<EPI_RESID>, grid, dim3(384), sm, p, ta, tb, ga);
    case EPI_GATED: return launch(e, gemm_wide_kernel<EPI_GATED>, grid, dim3(384), sm, p, ta, tb, ga);
    case EPI_GEGLU: return launch(e, gemm_wide_kernel<EPI_GEGLU>, grid, dim3(384), sm, p, ta, tb, ga);
    case EPI_F32: return launch(e, gemm_wide_kernel<EPI_F32>, grid, dim3(384), sm, p, ta, tb, ga);
    case EPI_ROPE: return launch(e, gemm_wide_kernel<EPI_ROPE>, grid, dim3(384), sm, p, ta, tb, ga);
    default: return launch(e, gemm_wide_kernel<EPI_STORE>, grid, dim3(384), sm, p, ta, tb, ga);
  }
}

bool set_gemm_wide_smem(pi05_engine* e) {
  const int sm = GemmWideCfg::SMEM;
  void (*k[])(CUtensorMap, CUtensorMap, GemmArgs) = {gemm_wide_kernel<EPI_STORE>, gemm_wide_kernel<EPI_GELU>,
                                                     gemm_wide_kernel<EPI_RESID>, gemm_wide_kernel<EPI_GATED>,
                                                     gemm_wide_kernel<EPI_GEGLU>, gemm_wide_kernel<EPI_F32>,
                                                     gemm_wide_kernel<EPI_ROPE>};
  for (auto f : k) CK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  return true;
}

template <int BN>
bool launch_gemm_bn(pi05_engine* e, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga) {
  // persistent: at most one CTA per SM, each walks units blockIdx.x, +gridDim.x, ...
  const int units = ga.tiles_m * ga.tiles_n * ga.splits;
  dim3 grid(std::min(units, e->num_sms));
  const size_t sm = (size_t)GemmCfg<BN>::SMEM;
  switch (ga.epi) {
    case EPI_GELU: return launch(e, gemm_tc_kernel<BN, EPI_GELU>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_RESID: return launch(e, gemm_tc_kernel<BN, EPI_RESID>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_GATED: return launch(e, gemm_tc_kernel<BN, EPI_GATED>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_GEGLU: return launch(e, gemm_tc_kernel<BN, EPI_GEGLU>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_ROPE: return launch(e, gemm_tc_kernel<BN, EPI_ROPE>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_F32: return launch(e, gemm_tc_kernel<BN, EPI_F32>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_GEGLU_BWD:
      return launch(e, gemm_tc_kernel<BN, EPI_GEGLU_BWD>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    default: return launch(e, gemm_tc_kernel<BN, EPI_STORE>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
  }
}

template <typename... KArgs, typename... Args>
bool launch_cluster(pi05_engine* e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster, bool pdl,
                    Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = e->stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = (pdl && e->pdl) ? 1 : 0;
  lc.attrs = at;
  lc.numAttrs = 2;
  CK(cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...));
  e->launches++;
  return true;
}

// CTA-pair GEMM: one cluster of two CTAs per 256x256 tile, persistent over the tiles
bool launch_gemm_pair(pi05_engine* e, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga) {
  const dim3 grid(2 * std::min(ga.tiles_m * ga.tiles_n, e->pair_clusters));
  const size_t sm = (size_t)GemmPairCfg::SMEM;
  const bool p = ga.pdl != 0;
  switch (ga.epi) {
    case EPI_GELU: return launch_cluster(e, gemm_pair_kernel<EPI_GELU>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_RESID: return launch_cluster(e, gemm_pair_kernel<EPI_RESID>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_GATED: return launch_cluster(e, gemm_pair_kernel<EPI_GATED>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_GEGLU: return launch_cluster(e, gemm_pair_kernel<EPI_GEGLU>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_ROPE: return launch_cluster(e, gemm_pair_kernel<EPI_ROPE>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_F32: return launch_cluster(e, gemm_pair_kernel<EPI_F32>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    case EPI_GEGLU_BWD:
      return launch_cluster(e, gemm_pair_kernel<EPI_GEGLU_BWD>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
    default: return launch_cluster(e, gemm_pair_kernel<EPI_STORE>, grid, dim3(GemmPairCfg::THREADS), sm, 2, p, ta, tb, ga);
  }
}

bool set_gemm_pair_smem(pi05_engine* e) {
  const int sm = GemmPairCfg::SMEM;
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_GATED>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_GEGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_pair_kernel<EPI_GEGLU_BWD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  // the persistent grid holds as many pairs as can be resident at once (pairs need two SMs of one GPC)
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(2 * (e->num_sms / 2));
  lc.blockDim = dim3(GemmPairCfg::THREADS);
  lc.dynamicSmemBytes = sm;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  int n = 0;
  CK(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI_STORE>, &lc));
  e->pair_clusters = std::min(n, e->num_sms / 2);
  if (e->pair_clusters < 1) e->gemm_pair = false;
  return true;
}

template <int BN>
bool launch_swap_cluster(pi05_engine* e, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga, int S) {
  const dim3 grid(ga.tiles_m * ga.tiles_n * S);
  const size_t sm = (size_t)GemmCfg<BN>::SMEM + SWAP_NRM_BYTES;
  const bool p = ga.pdl != 0;
  switch (ga.epi) {
    case EPI_GELU: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_GELU>, grid, dim3(256), sm, S, p, ta, tb, ga);
    case EPI_RESID: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_RESID>, grid, dim3(256), sm, S, p, ta, tb, ga);
    case EPI_GATED: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_GATED>, grid, dim3(256), sm, S, p, ta, tb, ga);
    case EPI_GEGLU: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_GEGLU>, grid, dim3(256), sm, S, p, ta, tb, ga);
    case EPI_ROPE: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_ROPE>, grid, dim3(256), sm, S, p, ta, tb, ga);
    case EPI_F32: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_F32>, grid, dim3(256), sm, S, p, ta, tb, ga);
    default: return launch_cluster(e, gemm_swap_cluster_kernel<BN, EPI_STORE>, grid, dim3(256), sm, S, p, ta, tb, ga);
  }
}

template <int BN>
bool set_swap_cluster_smem(pi05_engine* e) {
  const int sm = GemmCfg<BN>::SMEM + SWAP_NRM_BYTES;
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_GATED>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_GEGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_swap_cluster_kernel<BN, EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  return true;
}

template <int BN>
bool launch_gemm_small(pi05_engine* e, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga, bool amn) {
  const int units = ga.tiles_m * ga.tiles_n * ga.splits;
  dim3 grid(std::min(units, e->num_sms));
  const size_t sm = (size_t)GemmCfg<BN>::SMEM;
  if (amn) return launch(e, gemm_tc_kernel<BN, EPI_LORA_GRAD, true>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
  switch (ga.epi) {
    case EPI_STORE_T:
      return launch(e, gemm_tc_kernel<BN, EPI_STORE_T>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_LORA_GRAD:
      return launch(e, gemm_tc_kernel<BN, EPI_LORA_GRAD>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    case EPI_F32: return launch(e, gemm_tc_kernel<BN, EPI_F32>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
    default: return launch(e, gemm_tc_kernel<BN, EPI_STORE>, grid, dim3(256), sm, ga.pdl != 0, ta, tb, ga);
  }
}

template <int BN>
bool set_gemm_smem_small(pi05_engine* e) {
  const int sm = GemmCfg<BN>::SMEM;
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_LORA_GRAD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_STORE_T>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_LORA_GRAD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  return true;
}

template <int BN>
bool set_gemm_smem(pi05_engine* e) {
  const int sm = GemmCfg<BN>::SMEM;
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_GATED>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_GEGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_GEGLU_BWD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
  return true;
}

// Few M-tiles in the normal orientation (a few hundred to ~1000 tokens, e.g. SigLIP's 768 and Gemma's
// 968 at batch 1): put the weights on the 128-row side with up to 256 tokens per tile and split K over
// a cluster (on-chip reduction), when the normal tiling would leave more than half the SMs idle.
int wide_swap_split(pi05_engine* e, const Lin& L) {
  const int kt = (L.K + 63) / 64;
  const bool epi_ok = L.epi == EPI_STORE || L.epi == EPI_GELU || L.epi == EPI_RESID || L.epi == EPI_GATED ||
                      L.epi == EPI_GEGLU || L.epi == EPI_F32 || L.epi == EPI_ROPE;
  // measured: it pays for long K only (SigLIP fc2 K=4304: 26.8 -> 22.0 µs; Gemma down K=16384: 78.3 -> 74.7 µs),
  // and loses for K <= 2048 (the 128x256 partial tiles' DSMEM reduce costs more than the shorter K loop saves)
  if (!e->wide_swap || !e->cluster_splitk || L.T <= 128 || L.amn || !epi_ok || L.addend || L.out_t || kt < 64 ||
      L.epi == EPI_GEGLU_BWD)
    return 0;
  const int t256 = ((L.T + 127) / 128) * ((L.F + 255) / 256);
  if (t256 >= e->num_sms / 2) return 0;
  const int tiles = ((L.F + 127) / 128) * ((L.T + 255) / 256);
  const int want = std::min(8, std::min(e->num_sms / std::max(1, tiles), kt / 2));
  int S = 1;
  while (S * 2 <= want) S *= 2;
  return S >= 2 ? S : 0;
}

bool linear(pi05_engine* e, const Lin& L) {
  GemmArgs ga = {};
  const int wide_S = wide_swap_split(e, L);
  const bool swap = (L.T <= 128 && !L.no_swap && !L.amn) || wide_S > 0;
  int BN;
  CUtensorMap ta, tb;
  const int kt = (L.K + 63) / 64;
  int nsplit = 0;  // > 0: split count chosen with the tile width (non-swapped orientation)
  if (L.F <= 48 && !swap) {
    // small-N GEMMs of the LoRA path: U = x A^T, V = dy B, and the weight gradients (N = 16 per adapter)
    BN = (L.F + 15) / 16 * 16;
    ga.M = L.T;
    ga.N = L.F;
    ga.tiles_m = (L.T + 127) / 128;
    ga.tiles_n = 1;
    if (L.amn) {
      if (!make_tmap_box(e, &ta, L.x, L.K, L.T, L.ldx, 64, 64)) return false;
    } else if (!make_tmap(e, &ta, L.x, L.T, L.K, L.ldx, 128)) {
      return false;
    }
    if (!make_tmap(e, &tb, L.w, L.F, L.K, L.ldw, BN)) return false;
  } else if (L.amn) {
    return set_err(e, "MN-major A operand is only wired for N <= 48");
  } else if (swap) {
    BN = L.T <= 64 ? 64 : (L.T <= 128 ? 128 : 256);
    ga.M = L.F;
    ga.N = L.T;
    ga.tiles_m = (L.F + 127) / 128;
    ga.tiles_n = (L.T + BN - 1) / BN;
    if (!make_tmap(e, &ta, L.w, L.F, L.K, L.ldw, 128) || !make_tmap(e, &tb, L.x, L.T, L.K, L.ldx, BN)) return false;
  } else {
    // Measured on B200: the mainloop is bound by L2->shared-memory bandwidth, and a 128x256 tile
    // loads 25% fewer bytes per MAC than 128x128, so BN=256 wins unless it leaves more than half of
    // the SMs idle.  Split-K (partials through global memory) only pays for long K with few tiles.
    const int tm = (L.T + 127) / 128;
    const int t256 = tm * ((L.F + 255) / 256);
    if (t256 >= e->num_sms / 2) {
      BN = 256;
      nsplit = 1;
    } else if (kt >= 128 && 2 * t256 <= e->num_sms) {
      BN = 256;
      nsplit = 2;
    } else {
      BN = 128;
      nsplit = 1;
    }
    ga.M = L.T;
    ga.N = L.F;
    ga.tiles_m = tm;
    ga.tiles_n = (L.F + BN - 1) / BN;
    if (!make_tmap(e, &ta, L.x, L.T, L.K, L.ldx, 128) || !make_tmap(e, &tb, L.w, L.F, L.K, L.ldw, BN)) return false;
  }
  ga.K = L.K;
  ga.swap = swap;
  // Tile order: walk all N-tiles for a group of M-tiles whose A rows (~48 MB) stay in L2, so the
  // weights are streamed from HBM once per group.
  ga.group_m = swap ? 1 : std::max(1, std::min(ga.tiles_m, (int)((48ull << 20) / (128ull * L.K * 2))));
  const int tiles = ga.tiles_m * ga.tiles_n;
  int splits = 1;
  if (nsplit > 0) {
    splits = nsplit;
    while (splits > 1 && ((size_t)splits * tiles * 128 * BN * 4 > e->gemm_ws_bytes || tiles > e->n_counters)) --splits;
  } else if (tiles < e->num_sms && kt >= 4) {
    splits = std::max(1, std::min(e->num_sms / tiles, kt / 2));
    const size_t need = (size_t)splits * tiles * 128 * BN * 4;
    while (splits > 1 && ((size_t)splits * tiles * 128 * BN * 4 > e->gemm_ws_bytes || tiles > e->n_counters)) --splits;
    (void)need;
  }
  int kper = (kt + splits - 1) / splits;
  splits = (kt + kper - 1) / kper;  // no empty split
  ga.splits = splits;
  ga.kt_per_split = kper;
  ga.epi = L.epi;
  ga.out = L.out;
  ga.ld_out = L.ld_out;
  ga.out_f32 = L.out_f32;
  ga.ld_out_f32 = L.ld_out_f32;
  ga.bias = L.bias;
  ga.res = L.res;
  ga.ld_res = L.ld_res;
  ga.gate = L.gate;
  ga.ld_gate = L.ld_gate;
  ga.gate_div = L.gate_div;
  ga.out_scale = L.out_scale;
  ga.addend = L.addend;
  ga.add_ld = L.add_ld;
  ga.add_mod = L.add_mod;
  ga.ws = e->gemm_ws;
  ga.counters = e->counters;
  ga.status = e->d_status;
  ga.pdl = e->pdl ? 1 : 0;
  ga.out_t = L.out_t;
  ga.ld_out_t = L.ld_out_t;
  ga.rope_cos = L.rope_cos;
  ga.rope_sin = L.rope_sin;
  ga.rope_pos_off = L.rope_pos_off;
  ga.rope_base = L.rope_base;
  ga.rope_per_sample = L.rope_per_sample;
  ga.rope_ld_kv = L.rope_ld_kv;
  ga.rope_k = L.rope_k;
  ga.rope_v = L.rope_v;
  ga.lg_mode = L.lg_mode;
  ga.lg_trans = L.lg_trans;
  ga.lg_K = L.lg_K;
  for (int i = 0; i < 3; ++i) ga.lg_off[i] = L.lg_off[i];
  ga.nrm_ss = L.nrm_ss;
  ga.nrm_ss_ld = L.nrm_ss_ld;
  ga.nrm_parts = L.nrm_parts;
  ga.nrm_D = L.nrm_D;
  ga.nrm_scale = L.nrm_scale;
  ga.nrm_shift = L.nrm_shift;
  ga.ss_out = L.ss_out;
  ga.ss_ld = L.ss_ld;
  const bool fused_nrm = L.nrm_ss || L.ss_out;
  if (swap && (splits > 1 || wide_S > 0) && e->cluster_splitk) {
    // few tokens, K split: reduce the split partials on chip inside a cluster of S CTAs
    int S = wide_S;
    if (S == 0) {
      S = 1;
      const int want = std::min(8, std::max(1, std::min(e->num_sms / ga.tiles_m, kt / 2)));
      while (S * 2 <= want) S *= 2;
    }
    if (S > 1) {
      ga.kt_per_split = (kt + S - 1) / S;
      ga.splits = S;
      if (L.nrm_ss && (BN != 64 || L.K % 64 != 0 || ga.kt_per_split * 64 > SWAP_NRM_KMAX || L.T > L.nrm_ss_ld ||
                       L.nrm_parts % 2 != 0 || ((uintptr_t)L.nrm_scale | (uintptr_t)L.nrm_shift) % 16 != 0))
        return set_err(e, "fused adaRMSNorm: unsupported shape");
      if (L.ss_out && (L.epi != EPI_GATED || S > 8 || L.F % 16 != 0 || L.T > L.ss_ld))
        return set_err(e, "sum-of-squares output: unsupported shape");
      return BN == 64    ? launch_swap_cluster<64>(e, ta, tb, ga, S)
             : BN == 128 ? launch_swap_cluster<128>(e, ta, tb, ga, S)
                         : launch_swap_cluster<256>(e, ta, tb, ga, S);
    }
  }
  if (L.epi == EPI_ROPE && swap) return set_err(e, "fused RoPE epilogue: few-token projection without a cluster split");
  if (L.epi == EPI_GEGLU_BWD && (swap || L.F % 32 || BN < 64 || L.ld_res % 8 || L.ld_out % 8 ||
                                 ((uintptr_t)L.res | (uintptr_t)L.out) % 16))
    return set_err(e, "fused GeGLU backward: normal orientation, F % 32 == 0, 16-byte aligned rows only");
  if (fused_nrm) return set_err(e, "fused adaRMSNorm / sum-of-squares output: not a few-token cluster projection");
  if (!swap && BN == 256 && splits == 1 && !L.amn && e->gemm_wide && L.epi != EPI_STORE_T && L.epi != EPI_LORA_GRAD &&
      L.epi != EPI_GEGLU_BWD && kt >= 64) {
    // at least a full wave of 256x256 tiles and K >= 4096: the wider tile loads a third fewer bytes per
    // MAC, but its single accumulator set leaves the epilogue unoverlapped, which only a long K loop
    // amortises (measured: Gemma down 3.67 -> 3.20 ms, SigLIP fc2 550 -> 451 µs at bs64; K = 2048
    // shapes 4-20 % slower)
    const int wtm = (L.T + 255) / 256, wtn = (L.F + 255) / 256;
    if ((long)wtm * wtn >= e->num_sms) {
      GemmArgs gw = ga;
      gw.tiles_m = wtm;
      gw.tiles_n = wtn;
      gw.splits = 1;
      gw.kt_per_split = kt;
      gw.group_m = std::max(1, std::min(wtm, (int)((48ull << 20) / (256ull * L.K * 2))));
      return launch_gemm_wide(e, ta, tb, gw);
    }
  }
  if (!swap && BN == 256 && splits == 1 && !L.amn && e->gemm_pair && L.epi != EPI_STORE_T &&
      L.epi != EPI_LORA_GRAD) {
    // one 256x256 tile per CTA pair: each SM stages half of A's and half of B's rows
    GemmArgs gp = ga;
    gp.tiles_m = (L.T + 255) / 256;
    gp.tiles_n = (L.F + 255) / 256;
    gp.group_m = std::max(1, std::min(gp.tiles_m, (int)((48ull << 20) / (256ull * L.K * 2))));
    CUtensorMap tb2;
    if (!make_tmap(e, &tb2, L.w, L.F, L.K, L.ldw, 128)) return false;
    return launch_gemm_pair(e, ta, tb2, gp);
  }
  if (BN == 16) return launch_gemm_small<16>(e, ta, tb, ga, L.amn);
  if (BN == 32) return launch_gemm_small<32>(e, ta, tb, ga, L.amn);
  if (BN == 48) return launch_gemm_small<48>(e, ta, tb, ga, L.amn);
  if (BN == 64) return launch_gemm_bn<64>(e, ta, tb, ga);
  if (BN == 128) return launch_gemm_bn<128>(e, ta, tb, ga);
  return launch_gemm_bn<256>(e, ta, tb, ga);
}

// head_dim-256 MQA attention on tcgen05 (attn_tc_kernel).  Splits the key tiles over CTAs when one
// CTA per 128-row block would leave SMs idle (never when the caller wants the log-sum-exp).
bool attention_tc(pi05_engine* e, const AttnArgs& a0, int batch) {
  using C = AttnTcCfg;
  AttnArgs a = a0;
  a.pdl = e->pdl ? 1 : 0;
  const int rows = a.T * 8, rb = (rows + C::ROWS - 1) / C::ROWS;
  const int ntiles = (a.len1 + C::KT - 1) / C::KT + (a.len2 + C::KT - 1) / C::KT;
  const long ctas = (long)rb * batch;
  int splits = 1;
  if (a.force_splits > 0) {
    splits = a.lse ? 1 : std::min(a.force_splits, ntiles);
  } else if (!a.lse && ctas < e->num_sms) {
    // waves x (tiles per CTA + ~2 tiles of fixed cost: Q load, epilogue); a split adds the fp32 partial
    // epilogue (~2 tiles) and the merge pass, whose traffic grows with rows x splits (measured in the
    // CUDA graph: 968-token prefix 15.10 -> 14.84 ms at bs1 without its 2 splits; the 50-token
    // expert keeps its 9)
    long best = -1;
    for (int s = 1; s <= std::min(ntiles, 16); ++s) {
      const int t = std::max((ntiles + s - 1) / s, s > 1 ? 2 : 1);
      const int se = (ntiles + t - 1) / t;
      const long merge = se > 1 ? 2 + (long)rows * se / 2048 : 0;
      const long cost = (ctas * se + e->num_sms - 1) / e->num_sms * (t + 2) + merge;
      if (best < 0 || cost < best) {
        best = cost;
        splits = se;
      }
    }
  }
  while (splits > 1 && (size_t)batch * splits * rows > e->attn_ws_rows) --splits;
  int tps = std::max((ntiles + splits - 1) / splits, splits > 1 ? 2 : 1);
  a.splits = std::max(1, (ntiles + tps - 1) / tps);
  if (a.splits == 1) tps = std::max(ntiles, 1);
  a.keys_per_split = tps * C::KT;
  if (a.splits > 1) {
    a.ws_o = e->attn_ws_o;
    a.ws_ml = e->attn_ws_ml;
    a.ws_half = e->attn_ws_half ? 1 : 0;
  }
  CUtensorMap tq, tk1, tv1, tk2, tv2;
  {
    const uint64_t dims[4] = {P5_HD, 8, (uint64_t)a.T, (uint64_t)batch};
    const uint64_t st[3] = {P5_HD * 2, (uint64_t)a.ldq * 2, (uint64_t)a.q_bstride * 2};
    const uint32_t box[4] = {64, 8, 16, 1};
    if (!make_tmap_nd(e, &tq, a.q, 4, dims, st, box)) return false;
  }
  auto kv_map = [&](CUtensorMap* m, const bf16* base, int len, int ld, long bstride) {
    const uint64_t dims[3] = {P5_HD, (uint64_t)len, (uint64_t)batch};
    const uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)bstride * 2};
    const uint32_t box[3] = {64, C::KT, 1};
    return make_tmap_nd(e, m, base, 3, dims, st, box);
  };
  if (!kv_map(&tk1, a.k1, a.len1, a.ld1, a.b1stride) || !kv_map(&tv1, a.v1, a.len1, a.ld1, a.b1stride)) return false;
  if (a.len2 > 0) {
    if (!kv_map(&tk2, a.k2, a.len2, a.ld2, a.b2stride) || !kv_map(&tv2, a.v2, a.len2, a.ld2, a.b2stride))
      return false;
  } else {
    tk2 = tk1;
    tv2 = tv1;
  }
  if (!launch(e, attn_tc_kernel, dim3(rb, 1, batch * a.splits), dim3(384), (size_t)C::SMEM, true, tq, tk1, tv1, tk2,
              tv2, a, e->d_status))
    return false;
  if (a.splits > 1) {
    const long n = (long)batch * rows * (P5_HD / 2);
    if (!launch(e, attn_combine_kernel<P5_HD>, dim3((n + 255) / 256), dim3(256), 0, true, a, batch)) return false;
  }
  return true;
}

bool attention(pi05_engine* e, const AttnArgs& a0, int batch, int hd) {
  if (hd == P5_HD && a0.G == 8 && a0.qdiv == 1.0f && e->attn_tc && a0.len1 > 0) return attention_tc(e, a0, batch);
  if (a0.valid1) return set_err(e, "the prompt padding mask needs the tensor-core attention (PI05_ATTN_TC=1)");
  if (a0.group1 > 0) return set_err(e, "prefix attention groups need the tensor-core attention (PI05_ATTN_TC=1)");
  // SigLIP: one CTA per (128 queries, head, image) on tcgen05 up to 32 images; measured per call (CUDA events,
  // 20 launches): 3 images 9.7 vs 14.5 us, 24 images 51.4 vs 55.5 us, 48 images 111.7 vs 101.3 us, 192 images
  // 422.8 vs 378.2 us for the tcgen05 and the mma.sync kernel, so the larger batches take the mma.sync kernel
  if (hd == P5_SIG_HD && a0.G == 1 && e->attn_tc && batch <= 32 && a0.T == AttnSigCfg::ROWS * 2 &&
      a0.len1 == AttnSigCfg::KEYS && a0.len2 == 0 && !a0.lse) {
    AttnArgs a = a0;
    a.pdl = e->pdl ? 1 : 0;
    return launch(e, attn_sig_kernel, dim3(2, P5_SIG_HEADS, batch), dim3(384), (size_t)AttnSigCfg::SMEM, true, a,
                  e->d_status);
  }
  AttnArgs a = a0;
  a.pdl = e->pdl ? 1 : 0;
  const int rows = a.T * a.G;
  const int total = a.len1 + a.len2;
  if (a.splits < 1) a.splits = 1;
  a.keys_per_split = ((total + a.splits - 1) / a.splits + 63) / 64 * 64;
  a.splits = (total + a.keys_per_split - 1) / a.keys_per_split;
  if (a.splits > 1) {
    if ((size_t)batch * a.splits * rows > e->attn_ws_rows) {
      a.splits = 1;
      a.keys_per_split = total;
    } else {
      a.ws_o = e->attn_ws_o;
      a.ws_ml = e->attn_ws_ml;
    }
  }
  const int heads = a.G == 1 ? (hd == P5_SIG_HD ? P5_SIG_HEADS : 1) : 1;
  // 8 warps (128 query rows share each K/V tile) when that still gives two waves of CTAs, else 4
  const bool wide = (long)((rows + 127) / 128) * heads * batch * a.splits >= 2L * e->num_sms;
  dim3 grid((rows + (wide ? 127 : 63)) / (wide ? 128 : 64), heads, batch * a.splits);
  if (hd == P5_HD) {
    const bool ok = wide ? launch(e, attn_kernel<P5_HD, 8>, grid, dim3(256), (size_t)AttnCfg<P5_HD, 8>::SMEM, true, a)
                         : launch(e, attn_kernel<P5_HD, 4>, grid, dim3(128), (size_t)AttnCfg<P5_HD, 4>::SMEM, true, a);
    if (!ok) return false;
    if (a.splits > 1) {
      const long n = (long)batch * rows * (P5_HD / 2);
      if (!launch(e, attn_combine_kernel<P5_HD>, dim3((n + 255) / 256), dim3(256), 0, true, a, batch)) return false;
    }
    return true;
  }
  return wide ? launch(e, attn_kernel<P5_SIG_HD, 8>, grid, dim3(256), (size_t)AttnCfg<P5_SIG_HD, 8>::SMEM, true, a)
              : launch(e, attn_kernel<P5_SIG_HD, 4>, grid, dim3(128), (size_t)AttnCfg<P5_SIG_HD, 4>::SMEM, true, a);
}

int rows_grid(long rows_warps) { return (int)((rows_warps * 32 + 255) / 256); }

// Verify run: wait for the stream, copy a [rows][cols] bf16 (ld-strided) or fp32 block of sample 0 to
// the host as fp32 and hand it to the probe callback.
// In a teacher-forced run the callback may overwrite the values, which are then written back (rounded to
// bf16 for bf16 points), so the kernels after this point start from them.
bool emit_bf16(pi05_engine* e, const std::string& name, const bf16* dev, long rows, int cols, int ld) {
  if (!e->probe_fn && !e->plant_fn) return true;
  std::vector<uint16_t> h((size_t)rows * cols);
  CK(cudaMemcpy2DAsync(h.data(), (size_t)cols * 2, dev, (size_t)ld * 2, (size_t)cols * 2, rows,
                       cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  std::vector<float> f(h.size());
  for (size_t i = 0; i < h.size(); ++i) f[i] = p5_bf2f(h[i]);
  if (e->probe_fn) {
    e->probe_fn(name.c_str(), f.data(), (int64_t)f.size(), e->probe_ctx);
    return true;
  }
  e->plant_fn(name.c_str(), f.data(), (int64_t)f.size(), e->probe_ctx);
  for (size_t i = 0; i < h.size(); ++i) h[i] = p5_f2bf(f[i]);
  CK(cudaMemcpy2DAsync(const_cast<bf16*>(dev), (size_t)ld * 2, h.data(), (size_t)cols * 2, (size_t)cols * 2, rows,
                       cudaMemcpyHostToDevice, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return true;
}

bool emit_f32(pi05_engine* e, const std::string& name, const float* dev, long n) {
  if (!e->probe_fn && !e->plant_fn) return true;
  std::vector<float> f((size_t)n);
  CK(cudaMemcpyAsync(f.data(), dev, (size_t)n * 4, cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  if (e->probe_fn) {
    e->probe_fn(name.c_str(), f.data(), (int64_t)n, e->probe_ctx);
    return true;
  }
  e->plant_fn(name.c_str(), f.data(), (int64_t)n, e->probe_ctx);
  CK(cudaMemcpyAsync(const_cast<float*>(dev), f.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return true;
}

// ------------------------------------------------------------------ forward passes
bool run_siglip(pi05_engine* e, int n) {
  const int T = n * e->cfg.n_cameras * P5_SIG_TOK, D = P5_SIG_W;
  Acts& A = e->A;
  {
    const long tot = (long)T * P5_SIG_KPAD;
    if (!launch(e, patchify_kernel, dim3((unsigned)std::min<long>((tot + 255) / 256, 65535)), dim3(256), 0, false,
                A.images + (size_t)e->s0 * e->cfg.n_cameras * P5_IMG * P5_IMG * 3, A.patches, n * e->cfg.n_cameras))
      return false;
  }
  {
    Lin L{A.patches, P5_SIG_KPAD, T, e->sig_stem_w, P5_SIG_KPAD, D, P5_SIG_KPAD};
    L.out = A.sx;
    L.ld_out = D;
    L.bias = e->sig_stem_b;
    L.out_scale = 1.0f / 255.0f;
    L.addend = e->sig_posemb;
    L.add_ld = D;
    L.add_mod = 256;
    if (!linear(e, L)) return false;
    if (!emit_bf16(e, "img.stem", A.sx, T, D, D)) return false;
  }
  for (int l = 0; l < e->cfg.siglip_layers; ++l) {
    const SigLayer& s = e->sig[l];
    if (!launch(e, layernorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.sx, A.sy, s.ln1s, s.ln1b, T, D))
      return false;
    Lin q{A.sy, D, T, s.wqkv, D, P5_SIG_QKV, D};
    q.out = A.sqkv;
    q.ld_out = P5_SIG_QKV;
    q.bias = s.bqkv;
    if (!linear(e, q)) return false;
    AttnArgs at = {};
    at.q = A.sqkv;
    at.ldq = P5_SIG_QKV;
    at.q_bstride = (long)256 * P5_SIG_QKV;
    at.out = A.so;
    at.ldo = D;
    at.o_bstride = (long)256 * D;
    at.k1 = A.sqkv + D;
    at.v1 = A.sqkv + 2 * D;
    at.ld1 = P5_SIG_QKV;
    at.len1 = 256;
    at.b1stride = (long)256 * P5_SIG_QKV;
    at.k2 = at.k1;
    at.v2 = at.v1;
    at.T = 256;
    at.G = 1;
    at.qdiv = P5_SIG_QDIV;
    at.splits = 1;
    if (!attention(e, at, n * e->cfg.n_cameras, P5_SIG_HD)) return false;
    Lin o{A.so, D, T, s.wo, D, D, D};
    o.epi = EPI_RESID;
    o.out = A.sx;
    o.ld_out = D;
    o.bias = s.bo;
    o.res = A.sx;
    o.ld_res = D;
    if (!linear(e, o)) return false;
    if (!launch(e, layernorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.sx, A.sy, s.ln2s, s.ln2b, T, D))
      return false;
    Lin m1{A.sy, D, T, s.w1, D, P5_SIG_MLP, D};
    m1.epi = EPI_GELU;
    m1.out = A.sh;
    m1.ld_out = P5_SIG_MLP;
    m1.bias = s.b1;
    if (!linear(e, m1)) return false;
    Lin m2{A.sh, P5_SIG_MLP, T, s.w2, P5_SIG_MLP, D, P5_SIG_MLP};
    m2.epi = EPI_RESID;
    m2.out = A.sx;
    m2.ld_out = D;
    m2.bias = s.b2;
    m2.res = A.sx;
    m2.ld_res = D;
    if (!linear(e, m2)) return false;
    if (!emit_bf16(e, "img.l" + std::to_string(l) + ".out", A.sx, T, D, D)) return false;
  }
  if (!launch(e, layernorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.sx, A.sy, e->sig_post_s, e->sig_post_b,
              T, D))
    return false;
  if (!emit_bf16(e, "img.encoded", A.sy, T, D, D)) return false;
  // projector 1152 -> 2048 straight into the image rows of each sample's prefix
  const int img_tok = e->cfg.n_cameras * P5_SIG_TOK;
  for (int b = 0; b < n; ++b) {
    Lin h{A.sy + (size_t)b * img_tok * D, D, img_tok, e->sig_head_w, D, P5_GEM_W, D};
    h.out = A.px + (size_t)b * e->P * P5_GEM_W;
    h.ld_out = P5_GEM_W;
    h.bias = e->sig_head_b;
    if (!linear(e, h)) return false;
  }
  return emit_bf16(e, "img.tokens", A.px, img_tok, P5_GEM_W, P5_GEM_W);
}

bool run_gemma(pi05_engine* e, int n) {
  const int P = e->P, T = n * P, D = P5_GEM_W;
  Acts& A = e->A;
  const size_t cache_layer = (size_t)e->max_batch * P * P5_HD;
  for (int l = 0; l < e->cfg.gemma_layers; ++l) {
    const GemLayer& g = e->gem[l];
    if (!launch(e, rmsnorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.px, A.ph, g.rms1, (const bf16*)nullptr,
                T, D, 1, 0, D))
      return false;
    const std::string pl = "pre.l" + std::to_string(l);
    if (!emit_bf16(e, pl + ".norm1", A.ph, P, D, D)) return false;
    bf16* kc = A.kcache + l * cache_layer + (size_t)e->s0 * P * P5_HD;
    bf16* vc = A.vcache + l * cache_layer + (size_t)e->s0 * P * P5_HD;
    // q/k/v projection with RoPE (and the K/V cache write) in the epilogue
    Lin q{A.ph, D, T, e->gem_wqkv_il + (size_t)l * P5_QKV * D, D, P5_QKV, D};
    q.epi = EPI_ROPE;
    q.no_swap = true;
    q.out = A.pqkv;
    q.ld_out = P5_QKV;
    q.rope_cos = e->d_cos;
    q.rope_sin = e->d_sin;
    q.rope_pos_off = 0;
    q.rope_per_sample = P;
    q.rope_ld_kv = P5_HD;
    q.rope_k = kc;
    q.rope_v = vc;
    if (!linear(e, q)) return false;
    if (!emit_bf16(e, pl + ".k", kc, P, P5_HD, P5_HD) || !emit_bf16(e, pl + ".v", vc, P, P5_HD, P5_HD)) return false;
    if (l == e->cfg.gemma_layers - 1) break;  // later outputs of the last layer feed nothing
    AttnArgs at = {};
    at.q = A.pqkv;
    at.ldq = P5_QKV;
    at.q_bstride = (long)P * P5_QKV;
    at.out = A.po;
    at.ldo = P5_QDIM;
    at.o_bstride = (long)P * P5_QDIM;
    at.k1 = kc;
    at.v1 = vc;
    at.ld1 = P5_HD;
    at.len1 = P;
    at.b1stride = (long)P * P5_HD;
    at.k2 = kc;
    at.v2 = vc;
    at.T = P;
    at.G = P5_NH;
    at.qdiv = 1.0f;
    at.splits = 1;
    at.valid1 = e->cfg.text_pad_mask ? e->d_valid + e->s0 : nullptr;
    at.group1 = e->cfg.prefix_group;
    if (!attention(e, at, n, P5_HD)) return false;
    Lin o{A.po, P5_QDIM, T, g.wo, P5_QDIM, D, P5_QDIM};
    o.epi = EPI_RESID;
    o.out = A.px;
    o.ld_out = D;
    o.res = A.px;
    o.ld_res = D;
    if (!linear(e, o)) return false;
    if (!launch(e, rmsnorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.px, A.ph, g.rms2, (const bf16*)nullptr,
                T, D, 1, 0, D))
      return false;
    if (!emit_bf16(e, pl + ".norm2", A.ph, P, D, D)) return false;
    Lin gu{A.ph, D, T, g.wgu, D, 2 * P5_GEM_MLP, D};
    gu.epi = EPI_GEGLU;
    gu.out = A.pact;
    gu.ld_out = P5_GEM_MLP;
    if (!linear(e, gu)) return false;
    Lin dn{A.pact, P5_GEM_MLP, T, g.wd, P5_GEM_MLP, D, P5_GEM_MLP};
    dn.epi = EPI_RESID;
    dn.out = A.px;
    dn.ld_out = D;
    dn.res = A.px;
    dn.ld_res = D;
    if (!linear(e, dn)) return false;
    if (!emit_bf16(e, pl + ".out", A.px, P, D, D)) return false;
  }
  return true;
}

bool run_prefill_body(pi05_engine* e, int n) {
  if (e->cfg.text_pad_mask &&
      !launch(e, text_valid_kernel, dim3((n + 127) / 128), dim3(128), 0, false,
              (const int32_t*)e->A.tokens + (size_t)e->s0 * e->cfg.n_text, n, e->cfg.n_text,
              e->cfg.n_cameras * P5_SIG_TOK, e->d_valid + e->s0))
    return false;
  if (!run_siglip(e, n)) return false;
  if (e->cfg.n_text > 0 && e->text_from_emb) {
    if (!launch(e, copy_text_emb_kernel, dim3(e->cfg.n_text, n), dim3(256), 0, true,
                (const bf16*)e->text_emb + (size_t)e->s0 * e->cfg.n_text * P5_GEM_W, e->A.px, e->cfg.n_text, e->P,
                e->cfg.n_cameras * P5_SIG_TOK))
      return false;
  } else if (e->cfg.n_text > 0 &&
      !launch(e, embed_text_kernel, dim3(e->cfg.n_text, n), dim3(256), 0, true,
              (const int32_t*)e->A.tokens + (size_t)e->s0 * e->cfg.n_text,
              (const bf16*)e->embed, e->A.px, e->cfg.n_text, e->P, e->cfg.n_cameras * P5_SIG_TOK))
    return false;
  if (e->cfg.n_text > 0 && !emit_bf16(e, "txt.emb", e->A.px + (size_t)e->cfg.n_cameras * P5_SIG_TOK * P5_GEM_W,
                                      e->cfg.n_text, P5_GEM_W, P5_GEM_W))
    return false;
  return run_gemma(e, n);
}

// The persistent one-sample denoise applies when a single sample's action tokens fit the N=64 side of
// its GEMM tiles and the GPU has enough SMs for every phase's units.
bool mega_applies(pi05_engine* e, int n) {
  const int H = e->cfg.horizon;
  const int attn_units = ((H * 8 + 127) / 128) * 9;
  return e->mega && n == 1 && H >= 1 && H <= 64 && e->cfg.expert_layers > 0 && e->num_sms >= 128 &&
         e->num_sms >= attn_units + 1 && e->P > 0;
}

// Expert q/k/v weights with interleaved head rows for the fused-RoPE projections, rebuilt whenever
// the weights changed.  Runs outside stream capture.
bool qkv_interleave_prepare(pi05_engine* e) {
  const int L = e->cfg.expert_layers, LG = e->cfg.gemma_layers;
  const size_t wq = (size_t)P5_QKV * P5_EXP_W, wg = (size_t)P5_QKV * P5_GEM_W;
  if (!e->exp_wqkv_il && !dalloc(e, (void**)&e->exp_wqkv_il, (size_t)std::max(L, 1) * wq * 2)) return false;
  if (!e->gem_wqkv_il && !dalloc(e, (void**)&e->gem_wqkv_il, (size_t)std::max(LG, 1) * wg * 2)) return false;
  if (e->qkv_il_wgen != e->wgen) {
    for (int l = 0; l < L; ++l)
      if (!launch(e, interleave_qkv_rows_kernel, dim3(P5_QKV), dim3(128), 0, false, (const bf16*)e->ex[l].wqkv,
                  e->exp_wqkv_il + l * wq, (int)P5_EXP_W))
        return false;
    for (int l = 0; l < LG; ++l)
      if (!launch(e, interleave_qkv_rows_kernel, dim3(P5_QKV), dim3(128), 0, false, (const bf16*)e->gem[l].wqkv,
                  e->gem_wqkv_il + l * wg, (int)P5_GEM_W))
        return false;
    e->qkv_il_wgen = e->wgen;
  }
  return true;
}

// The q/k/v projection of a denoise with n samples runs with RoPE fused: more than 64 tokens in the
// normal orientation, up to 64 through the on-chip cluster split-K path.
bool fused_rope_applies(pi05_engine* e, int n) {
  const int T = n * e->cfg.horizon;
  return T > 64 || e->cluster_splitk;  // > 64 tokens: normal orientation; <= 64: cluster split-K
}

// adaRMSNorm folded into the few-token q/k/v and gate/up cluster GEMMs (one 64-token tile)
bool fused_norm_applies(pi05_engine* e, int n) {
  const int T = n * e->cfg.horizon;
  // a teacher-forced run replaces the residual stream after the kernels that emit its sums of squares
  return e->fuse_norm && e->cluster_splitk && T <= 64 && P5_EXP_W % 32 == 0 && !e->plant_fn;
}

// Buffers and tensor-map table of the persistent denoise.  Runs outside stream capture.
bool mega_prepare(pi05_engine* e) {
  using C = MegaCfg;
  const int L = e->cfg.expert_layers, H = e->cfg.horizon, P = e->P;
  const size_t wq = (size_t)P5_QKV * P5_EXP_W;
  const int nmaps = L * C::NMAPS_LAYER + 5;
  if (!qkv_interleave_prepare(e)) return false;
  if (!e->mega_maps) {
    if (!dalloc(e, (void**)&e->mega_maps, (size_t)nmaps * sizeof(CUtensorMap)) ||
        !dalloc(e, (void**)&e->mega_ctr, MG_NCTR * 4))
      return false;
    Acts& A = e->A;
    const size_t cache_layer = (size_t)e->max_batch * P * P5_HD;
    std::vector<CUtensorMap> m(nmaps);
    auto kv3 = [&](CUtensorMap* t, const bf16* base, int len) {
      const uint64_t dims[3] = {P5_HD, (uint64_t)len, 1};
      const uint64_t st[2] = {P5_HD * 2, (uint64_t)len * P5_HD * 2};
      const uint32_t box[3] = {64, AttnTcCfg::KT, 1};
      return make_tmap_nd(e, t, base, 3, dims, st, box);
    };
    for (int l = 0; l < L; ++l) {
      CUtensorMap* t = &m[(size_t)l * C::NMAPS_LAYER];
      const ExpLayer& x = e->ex[l];
      if (!make_tmap(e, t + 0, e->exp_wqkv_il + l * wq, P5_QKV, P5_EXP_W, P5_EXP_W, 128) ||
          !make_tmap(e, t + 1, x.wo, P5_EXP_W, P5_QDIM, P5_QDIM, 128) ||
          !make_tmap(e, t + 2, x.wgu, 2 * P5_EXP_MLP, P5_EXP_W, P5_EXP_W, 128) ||
          !make_tmap(e, t + 3, x.wd, P5_EXP_W, P5_EXP_MLP, P5_EXP_MLP, 128) ||
          !kv3(t + 4, A.kcache + l * cache_layer, P) || !kv3(t + 5, A.vcache + l * cache_layer, P))
        return false;
    }
    CUtensorMap* g = &m[(size_t)L * C::NMAPS_LAYER];
    {
      const uint64_t dims[4] = {P5_HD, 8, (uint64_t)H, 1};
      const uint64_t st[3] = {P5_HD * 2, (uint64_t)P5_QKV * 2, (uint64_t)H * P5_QKV * 2};
      const uint32_t box[4] = {64, 8, 16, 1};
      if (!make_tmap_nd(e, g + 0, A.eqkv, 4, dims, st, box)) return false;
    }
    if (!kv3(g + 1, A.ek, H) || !kv3(g + 2, A.ev, H) || !make_tmap_box(e, g + 3, A.eo, H, P5_QDIM, P5_QDIM, 64, 64) ||
        !make_tmap_box(e, g + 4, A.eact, H, P5_EXP_MLP, P5_EXP_MLP, 64, 64))
      return false;
    CK(cudaMemcpyAsync(e->mega_maps, m.data(), m.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, e->stream));
  }
  return true;
}

bool run_denoise_mega(pi05_engine* e) {
  using C = MegaCfg;
  const int H = e->cfg.horizon;
  Acts& A = e->A;
  MegaArgs m = {};
  m.x = A.ex;
  m.xt = A.xt;
  m.qkv = A.eqkv;
  m.ek = A.ek;
  m.ev = A.ev;
  m.eo = A.eo;
  m.act = A.eact;
  m.ws = e->gemm_ws;
  m.attn_o = e->attn_ws_o;
  m.attn_ml = e->attn_ws_ml;
  m.attn_half = e->attn_ws_half ? 1 : 0;
  m.ctr = e->mega_ctr;
  m.status = e->d_status;
  m.mods = e->mods;
  m.ain_w = e->ain_w;
  m.ain_b = e->ain_b;
  m.aout_w = e->aout_w;
  m.aout_b = e->aout_b;
  m.cos_t = e->d_cos;
  m.sin_t = e->d_sin;
  m.maps = e->mega_maps;
  m.T = H;
  m.P = e->P;
  m.L = e->cfg.expert_layers;
  m.steps = e->cfg.num_steps;
  m.NM = e->NM;
  m.dtb = p5_dt_bf16(e->cfg.num_steps);
  const int ntiles = (e->P + AttnTcCfg::KT - 1) / AttnTcCfg::KT + (H + AttnTcCfg::KT - 1) / AttnTcCfg::KT;
  m.attn_tps = std::max(1, (ntiles + 8) / 9);
  m.attn_splits = (ntiles + m.attn_tps - 1) / m.attn_tps;
  if ((size_t)m.attn_splits * H * 8 > e->attn_ws_rows || (size_t)mg_units(MG_O) * 128 * 64 * 4 > e->gemm_ws_bytes)
    return set_err(e, "persistent denoise: workspace too small");
  CK(cudaMemsetAsync(e->mega_ctr, 0, MG_NCTR * 4, e->stream));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(e->num_sms);
  lc.blockDim = dim3(C::THREADS);
  lc.dynamicSmemBytes = C::SMEM;
  lc.stream = e->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid-wide barriers rely on it
  at[0].val.cooperative = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  CK(cudaLaunchKernelEx(&lc, denoise_mega_kernel, m));
  e->launches++;
  return true;
}

bool run_denoise_body(pi05_engine* e, int n) {
  if (mega_applies(e, n) && !e->probe_fn && !e->plant_fn && e->s0 == 0 && !e->cfg.text_pad_mask && !e->inp_fixed &&
      !e->kv_mix)
    return run_denoise_mega(e);
  const int H = e->cfg.horizon, T = n * H, D = P5_EXP_W, P = e->P;
  Acts& A = e->A;
  float* xt = A.xt + (size_t)e->s0 * H * P5_ACT_D;
  const size_t kv_s0 = (size_t)e->s0 * P * P5_HD;
  const size_t cache_layer = (size_t)e->max_batch * P * P5_HD;
  const int MW = e->NM * 3 * D;  // modulation row width
  const float dtb = p5_dt_bf16(e->cfg.num_steps);
  const int attn_splits = n <= 4 ? 8 : 1;
  // soft inpainting: the step-0 noise is kept, the flow time after step s is tsched[s + 1] (the same fp32
  // accumulation as the time conditioning's schedule)
  const int inp_k = e->inp_fixed * P5_ACT_D;
  std::vector<float> tsched(e->cfg.num_steps + 1);
  {
    const float dt = (float)(-1.0 / (double)e->cfg.num_steps);
    float t = 1.0f;
    for (int s = 0; s <= e->cfg.num_steps; ++s) {
      tsched[s] = t;
      t = t + dt;
    }
  }
  if (inp_k > 0)
    CK(cudaMemcpyAsync(e->inp_eps, xt, (size_t)T * P5_ACT_D * 4, cudaMemcpyDeviceToDevice, e->stream));
  // KV layer mixing: the mixed caches of this call's samples, once per denoise
  const bf16* kc = e->kv_mix ? e->kmix : A.kcache;
  const bf16* vc = e->kv_mix ? e->vmix : A.vcache;
  if (e->kv_mix) {
    const int L = e->cfg.gemma_layers;
    const long items = (long)n * P * (P5_HD / 8);
    const int LL = L * L;
    if (!launch(e, kv_mix_kernel, dim3((unsigned)((items + 127) / 128)), dim3(128), 0, false, (const bf16*)A.kcache,
                e->kmix, (const float*)e->mix_w, (const float*)e->mix_b, L, (long)cache_layer, (long)kv_s0, items) ||
        !launch(e, kv_mix_kernel, dim3((unsigned)((items + 127) / 128)), dim3(128), 0, false, (const bf16*)A.vcache,
                e->vmix, (const float*)(e->mix_w + LL), (const float*)(e->mix_b + (size_t)L * P5_HD), L,
                (long)cache_layer, (long)kv_s0, items))
      return false;
  }
  // fused adaRMSNorm: x's producers (action_in, O and down projections) write per-token sums of squares
  // over 16-feature groups; the q/k/v and gate/up projections read x and normalise it on chip
  const bool fnorm = fused_norm_applies(e, n);
  constexpr int NP = P5_EXP_W / 16, SSLD = 64;
  float* ss_attn = e->nrm_ss;              // written by O (x after attention), read by gate/up
  float* ss_mlp = e->nrm_ss + NP * SSLD;  // written by action_in / down (x after the MLP), read by q/k/v
  auto fuse = [&](Lin& L, const float* ss, const bf16* mod) {
    L.x = A.ex;
    L.nrm_ss = ss;
    L.nrm_ss_ld = SSLD;
    L.nrm_parts = NP;
    L.nrm_D = D;
    L.nrm_scale = mod;
    L.nrm_shift = mod + D;
  };
  for (int s = 0; s < e->cfg.num_steps; ++s) {
    const bf16* mrow = e->mods + (size_t)s * MW;
    if (!launch(e, action_in_kernel, dim3((T * D + 255) / 256), dim3(256), 0, true, (const float*)xt,
                (const bf16*)e->ain_w, (const bf16*)e->ain_b, A.ex, T, D, fnorm ? ss_mlp : (float*)nullptr, SSLD))
      return false;
    const std::string sp = "suf.s" + std::to_string(s);
    if (!emit_bf16(e, sp + ".in", A.ex, H, D, D)) return false;
    for (int l = 0; l < e->cfg.expert_layers; ++l) {
      const ExpLayer& x = e->ex[l];
      const bf16* m1 = mrow + (size_t)(2 * l) * 3 * D;
      const bf16* m2 = mrow + (size_t)(2 * l + 1) * 3 * D;
      if (!fnorm &&
          !launch(e, rmsnorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.ex, A.eh, m1, m1 + D, T, D, 1, 0, D))
        return false;
      if (fused_rope_applies(e, n)) {
        Lin q{A.eh, D, T, e->exp_wqkv_il + (size_t)l * P5_QKV * D, D, P5_QKV, D};
        if (fnorm) fuse(q, ss_mlp, m1);
        q.no_swap = T > 64;
        q.epi = EPI_ROPE;
        q.out = A.eqkv;
        q.ld_out = P5_QKV;
        q.rope_cos = e->d_cos;
        q.rope_sin = e->d_sin;
        q.rope_pos_off = P;
        q.rope_per_sample = H;
        if (e->cfg.text_pad_mask) q.rope_base = e->d_valid + e->s0;  // action tokens follow the real prompt
        q.rope_ld_kv = P5_HD;
        q.rope_k = A.ek;
        q.rope_v = A.ev;
        if (!linear(e, q)) return false;
      } else {
        Lin q{A.eh, D, T, x.wqkv, D, P5_QKV, D};
        q.out = A.eqkv;
        q.ld_out = P5_QKV;
        if (!linear(e, q)) return false;
        if (e->cfg.text_pad_mask)
          return set_err(e, "the prompt padding mask needs the fused RoPE projections (PI05_CLUSTER_SPLITK=1)");
        if (!launch(e, rope_qkv_kernel, dim3(T), dim3(256), 0, true, A.eqkv, T, H, P, A.ek, A.ev,
                    (const float*)e->d_cos, (const float*)e->d_sin, 256))
          return false;
      }
      AttnArgs at = {};
      at.q = A.eqkv;
      at.ldq = P5_QKV;
      at.q_bstride = (long)H * P5_QKV;
      at.out = A.eo;
      at.ldo = P5_QDIM;
      at.o_bstride = (long)H * P5_QDIM;
      at.k1 = kc + l * cache_layer + kv_s0;
      at.v1 = vc + l * cache_layer + kv_s0;
      at.ld1 = P5_HD;
      at.len1 = P;
      at.b1stride = (long)P * P5_HD;
      at.k2 = A.ek;
      at.v2 = A.ev;
      at.ld2 = P5_HD;
      at.len2 = H;
      at.b2stride = (long)H * P5_HD;
      at.T = H;
      at.G = P5_NH;
      at.qdiv = 1.0f;
      at.splits = attn_splits;
      at.valid1 = e->cfg.text_pad_mask ? e->d_valid + e->s0 : nullptr;
      if (!attention(e, at, n, P5_HD)) return false;
      Lin o{A.eo, P5_QDIM, T, x.wo, P5_QDIM, D, P5_QDIM};
      o.epi = EPI_GATED;
      o.out = A.ex;
      o.ld_out = D;
      o.res = A.ex;
      o.ld_res = D;
      o.gate = m1 + 2 * D;
      o.ld_gate = 0;
      o.gate_div = 1;
      if (fnorm) {
        o.ss_out = ss_attn;
        o.ss_ld = SSLD;
      }
      if (!linear(e, o)) return false;
      if (!fnorm &&
          !launch(e, rmsnorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.ex, A.eh, m2, m2 + D, T, D, 1, 0, D))
        return false;
      Lin gu{A.eh, D, T, x.wgu, D, 2 * P5_EXP_MLP, D};
      if (fnorm) fuse(gu, ss_attn, m2);
      gu.epi = EPI_GEGLU;
      gu.out = A.eact;
      gu.ld_out = P5_EXP_MLP;
      if (!linear(e, gu)) return false;
      Lin dn{A.eact, P5_EXP_MLP, T, x.wd, P5_EXP_MLP, D, P5_EXP_MLP};
      dn.epi = EPI_GATED;
      dn.out = A.ex;
      dn.ld_out = D;
      dn.res = A.ex;
      dn.ld_res = D;
      dn.gate = m2 + 2 * D;
      dn.ld_gate = 0;
      dn.gate_div = 1;
      if (fnorm && l + 1 < e->cfg.expert_layers) {
        dn.ss_out = ss_mlp;
        dn.ss_ld = SSLD;
      }
      if (!linear(e, dn)) return false;
      if (!emit_bf16(e, sp + ".l" + std::to_string(l) + ".out", A.ex, H, D, D)) return false;
    }
    const bf16* mf = mrow + (size_t)(e->NM - 1) * 3 * D;
    if (!launch(e, rmsnorm_kernel, dim3(rows_grid(T)), dim3(256), 0, true, A.ex, A.eh, mf, mf + D, T, D, 1, 0, D))
      return false;
    if (!emit_bf16(e, sp + ".final", A.eh, H, D, D)) return false;
    // the verify run also keeps the velocity v (A.actions is otherwise unused scratch of this size)
    if (!launch(e, action_out_euler_kernel, dim3(rows_grid((long)T * P5_ACT_D)), dim3(256), 0, true,
                (const bf16*)A.eh, (const bf16*)e->aout_w, (const bf16*)e->aout_b, xt,
                (e->probe_fn || e->plant_fn) ? A.actions : (float*)nullptr, T, D, dtb))
      return false;
    if (inp_k > 0 && tsched[s] > e->inp_tmin &&
        !launch(e, inpaint_kernel, dim3(n), dim3(1024), (size_t)inp_k * 4, false, xt, (const float*)e->inp_eps,
                (const float*)e->inp_known, (const int*)e->inp_on, (const float*)e->inp_corr, e->s0, H, inp_k,
                tsched[s + 1]))
      return false;
    if (!emit_f32(e, sp + ".v", A.actions, (long)H * P5_ACT_D) || !emit_f32(e, sp + ".x", xt, (long)H * P5_ACT_D))
      return false;
  }
  return true;
}

// Capture `body` once per batch size n (and single-sample position s0) and replay it.
bool run_graph(pi05_engine* e, std::map<int, cudaGraphExec_t>& cache, std::map<int, long>& counts, int n,
               bool (*body)(pi05_engine*, int)) {
  const int key = n + (e->s0 << 16);
  auto it = cache.find(key);
  if (it == cache.end()) {
    cudaGraph_t g = nullptr;
    const long before = e->launches;
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const bool ok = body(e, n);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (!ok) {
      if (g) cudaGraphDestroy(g);
      return false;
    }
    if (ce != cudaSuccess) return set_err(e, std::string("graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return set_err(e, std::string("graph instantiate: ") + cudaGetErrorString(ce));
    counts[key] = e->launches - before;
    it = cache.emplace(key, ex).first;
  }
  CK(cudaGraphLaunch(it->second, e->stream));
  return true;
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

bool copy_in(pi05_engine* e, void* dst, const void* src, size_t bytes) {
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, e->stream));
  return true;
}

bool check_status(pi05_engine* e) {
  int st = 0;
  CK(cudaMemcpy(&st, e->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st != 0) {
    CK(cudaMemset(e->d_status, 0, sizeof(int)));
    return set_err(e, "device-side wait gave up (status " + std::to_string(st) + ")");
  }
  return true;
}

int fail_code(pi05_engine* e) {
  return e->err.rfind("device-side", 0) == 0 ? PI05_ERR_DEVICE : PI05_ERR_CUDA;
}

// Prefill of batch positions [0, n) whose images and tokens are already in A.images / A.tokens.  In
// batch-invariant mode every position runs the single-sample graph (at its own offsets), so a sample's
// result does not depend on the batch it came in.
bool prefill_resident(pi05_engine* e, int n) {
  if (!qkv_interleave_prepare(e)) return false;
  auto& graphs = e->text_from_emb ? e->prefill_emb_graphs : e->prefill_graphs;
  auto& launches = e->text_from_emb ? e->prefill_emb_launches : e->prefill_launches;
  if (!e->cfg.batch_invariant) return run_graph(e, graphs, launches, n, run_prefill_body);
  for (int b = 0; b < n; ++b) {
    e->s0 = b;
    const bool ok = run_graph(e, graphs, launches, 1, run_prefill_body);
    e->s0 = 0;
    if (!ok) return false;
  }
  return true;
}

// Denoise of batch positions [0, n) from the noise already in A.xt (the chunk replaces it there).
bool denoise_resident(pi05_engine* e, int n) {
  const int nb = e->cfg.batch_invariant ? 1 : n;
  if (mega_applies(e, nb) && !mega_prepare(e)) return false;
  if (fused_rope_applies(e, nb) && !qkv_interleave_prepare(e)) return false;
  if (!e->cfg.batch_invariant) return run_graph(e, e->denoise_graphs, e->denoise_launches, n, run_denoise_body);
  for (int b = 0; b < n; ++b) {
    e->s0 = b;
    const bool ok = run_graph(e, e->denoise_graphs, e->denoise_launches, 1, run_denoise_body);
    e->s0 = 0;
    if (!ok) return false;
  }
  return true;
}

// A prefix cache installed directly (not by a prefill) has no padding: every key of it is attended to.
bool set_valid_full(pi05_engine* e, int n) {
  std::vector<int> v(n, e->P);
  CK(cudaMemcpy(e->d_valid, v.data(), n * sizeof(int), cudaMemcpyHostToDevice));
  return true;
}

// Device buffer that grows to `need` bytes (contents are not kept).
bool grow(pi05_engine* e, void** p, size_t* cap, size_t need) {
  if (need <= *cap) return true;
  if (*p) {
    CK(cudaStreamSynchronize(e->stream));
    CK(cudaFree(*p));
    e->allocs.erase(std::find(e->allocs.begin(), e->allocs.end(), *p));
    *p = nullptr;
    *cap = 0;
  }
  const size_t bytes = need + need / 4;
  if (!dalloc(e, p, bytes)) return false;
  *cap = bytes;
  return true;
}

// time conditioning -> modulation table for every step (depends only on the fixed schedule)
bool build_mods(pi05_engine* e) {
  const int S = e->cfg.num_steps, D = P5_EXP_W;
  std::vector<float> ts(S), emb((size_t)S * D);
  p5_time_schedule(S, ts.data());
  for (int s = 0; s < S; ++s) p5_time_embedding(ts[s], D, emb.data() + (size_t)s * D);
  float *d_emb, *d_c1, *d_c2;
  bf16* d_cbf;
  CK(cudaMalloc(&d_emb, (size_t)S * D * 4));
  CK(cudaMalloc(&d_c1, (size_t)S * D * 4));
  CK(cudaMalloc(&d_c2, (size_t)S * D * 4));
  CK(cudaMalloc(&d_cbf, (size_t)S * D * 2));
  CK(cudaMemcpyAsync(d_emb, emb.data(), (size_t)S * D * 4, cudaMemcpyHostToDevice, e->stream));
  const int warps = S * D;
  linear_swish_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, e->stream>>>(d_emb, e->tin_w, e->tin_b, d_c1,
                                                                          (bf16*)nullptr, S, D);
  linear_swish_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, e->stream>>>(d_c1, e->tout_w, e->tout_b, d_c2, d_cbf,
                                                                          S, D);
  CK(cudaGetLastError());
  Lin m{d_cbf, D, S, e->ada_w, D, e->NM * 3 * D, D};
  m.out = e->mods;
  m.ld_out = e->NM * 3 * D;
  m.bias = e->ada_b;
  const bool ok = linear(e, m);
  CK(cudaStreamSynchronize(e->stream));
  cudaFree(d_emb);
  cudaFree(d_c1);
  cudaFree(d_c2);
  cudaFree(d_cbf);
  return ok && check_status(e);
}

struct Fill {
  bf16* dst;
  long rows;
  int cols, ld;
  long row_off;
  int row_step;
  int kind, sub;
  double stdv;
};

bool fill(pi05_engine* e, uint64_t seed, const Fill& f) {
  const uint64_t key = p5_key(seed, (uint32_t)f.kind, (uint32_t)f.sub);
  const float sc = p5_scale_for_std(f.stdv);
  const float base = p5_kind_has_unit_base(f.kind) ? 1.0f : 0.0f;
  const long n = f.rows * f.cols;
  const unsigned blocks = (unsigned)std::min<long>((n + 255) / 256, 148L * 64);
  fill_param_kernel<<<blocks, 256, 0, e->stream>>>(f.dst, f.rows, f.cols, f.ld, f.row_off, f.row_step, key, sc, base);
  CK(cudaGetLastError());
  return true;
}

bool init_random(pi05_engine* e, uint64_t seed) {
  const pi05_config& c = e->cfg;
  const double S = P5_W_STD;
  CK(cudaMemsetAsync(e->warena, 0, e->wbytes, e->stream));
  std::vector<Fill> F;
  const int D = P5_SIG_W;
  F.push_back({e->sig_stem_w, D, P5_SIG_K, P5_SIG_KPAD, 0, 1, K_SIG_STEM_W, 0, S});
  F.push_back({e->sig_stem_b, 1, D, D, 0, 1, K_SIG_STEM_B, 0, S});
  F.push_back({e->sig_posemb, 256, D, D, 0, 1, K_SIG_POSEMB, 0, S});
  for (int l = 0; l < c.siglip_layers; ++l) {
    const SigLayer& s = e->sig[l];
    F.push_back({s.ln1s, 1, D, D, 0, 1, K_SIG_LN1_S, l, S});
    F.push_back({s.ln1b, 1, D, D, 0, 1, K_SIG_LN1_B, l, S});
    F.push_back({s.wqkv, D, D, D, 0, 1, K_SIG_WQ, l, S});
    F.push_back({s.wqkv, D, D, D, D, 1, K_SIG_WK, l, S});
    F.push_back({s.wqkv, D, D, D, 2 * D, 1, K_SIG_WV, l, S});
    F.push_back({s.bqkv, 1, D, D, 0, 1, K_SIG_BQ, l, S});
    F.push_back({s.bqkv + D, 1, D, D, 0, 1, K_SIG_BK, l, S});
    F.push_back({s.bqkv + 2 * D, 1, D, D, 0, 1, K_SIG_BV, l, S});
    F.push_back({s.wo, D, D, D, 0, 1, K_SIG_WO, l, S});
    F.push_back({s.bo, 1, D, D, 0, 1, K_SIG_BO, l, S});
    F.push_back({s.ln2s, 1, D, D, 0, 1, K_SIG_LN2_S, l, S});
    F.push_back({s.ln2b, 1, D, D, 0, 1, K_SIG_LN2_B, l, S});
    F.push_back({s.w1, P5_SIG_MLP, D, D, 0, 1, K_SIG_W1, l, S});
    F.push_back({s.b1, 1, P5_SIG_MLP, P5_SIG_MLP, 0, 1, K_SIG_B1, l, S});
    F.push_back({s.w2, D, P5_SIG_MLP, P5_SIG_MLP, 0, 1, K_SIG_W2, l, S});
    F.push_back({s.b2, 1, D, D, 0, 1, K_SIG_B2, l, S});
  }
  F.push_back({e->sig_post_s, 1, D, D, 0, 1, K_SIG_POST_S, 0, S});
  F.push_back({e->sig_post_b, 1, D, D, 0, 1, K_SIG_POST_B, 0, S});
  F.push_back({e->sig_head_w, P5_GEM_W, D, D, 0, 1, K_SIG_HEAD_W, 0, S});
  F.push_back({e->sig_head_b, 1, P5_GEM_W, P5_GEM_W, 0, 1, K_SIG_HEAD_B, 0, S});
  F.push_back({e->embed, P5_VOCAB, P5_GEM_W, P5_GEM_W, 0, 1, K_GEM_EMBED, 0, S});
  const int G = P5_GEM_W;
  for (int l = 0; l < c.gemma_layers; ++l) {
    const GemLayer& g = e->gem[l];
    F.push_back({g.rms1, 1, G, G, 0, 1, K_GEM_RMS1, l, S});
    F.push_back({g.wqkv, P5_QDIM, G, G, 0, 1, K_GEM_WQ, l, S});
    F.push_back({g.wqkv, P5_HD, G, G, P5_QDIM, 1, K_GEM_WK, l, S});
    F.push_back({g.wqkv, P5_HD, G, G, P5_QDIM + P5_HD, 1, K_GEM_WV, l, S});
    F.push_back({g.wo, G, P5_QDIM, P5_QDIM, 0, 1, K_GEM_WO, l, S});
    F.push_back({g.rms2, 1, G, G, 0, 1, K_GEM_RMS2, l, S});
    F.push_back({g.wgu, P5_GEM_MLP, G, G, 0, 2, K_GEM_WG, l, S});  // gate rows even
    F.push_back({g.wgu, P5_GEM_MLP, G, G, 1, 2, K_GEM_WU, l, S});  // up rows odd
    F.push_back({g.wd, G, P5_GEM_MLP, P5_GEM_MLP, 0, 1, K_GEM_WD, l, S});
  }
  const int X = P5_EXP_W;
  for (int l = 0; l < c.expert_layers; ++l) {
    const ExpLayer& x = e->ex[l];
    F.push_back({x.wqkv, P5_QDIM, X, X, 0, 1, K_EXP_WQ, l, S});
    F.push_back({x.wqkv, P5_HD, X, X, P5_QDIM, 1, K_EXP_WK, l, S});
    F.push_back({x.wqkv, P5_HD, X, X, P5_QDIM + P5_HD, 1, K_EXP_WV, l, S});
    F.push_back({x.wo, X, P5_QDIM, P5_QDIM, 0, 1, K_EXP_WO, l, S});
    F.push_back({x.wgu, P5_EXP_MLP, X, X, 0, 2, K_EXP_WG, l, S});
    F.push_back({x.wgu, P5_EXP_MLP, X, X, 1, 2, K_EXP_WU, l, S});
    F.push_back({x.wd, X, P5_EXP_MLP, P5_EXP_MLP, 0, 1, K_EXP_WD, l, S});
  }
  for (int m = 0; m < e->NM; ++m) {
    const bool fin = m == e->NM - 1;
    const int kw = fin ? K_EXP_FINAL_W : ((m & 1) ? K_EXP_ADA2_W : K_EXP_ADA1_W);
    const int l = fin ? 0 : m / 2;
    F.push_back({e->ada_w, 3 * X, X, X, (long)m * 3 * X, 1, kw, l, S});
    F.push_back({e->ada_b + (size_t)m * 3 * X, 1, 3 * X, 3 * X, 0, 1, kw + 1, l, S});
  }
  F.push_back({e->ain_w, X, P5_ACT_D, P5_ACT_D, 0, 1, K_AIN_W, 0, S});
  F.push_back({e->ain_b, 1, X, X, 0, 1, K_AIN_B, 0, S});
  F.push_back({e->aout_w, P5_ACT_D, X, X, 0, 1, K_AOUT_W, 0, S});
  F.push_back({e->aout_b, 1, P5_ACT_D, P5_ACT_D, 0, 1, K_AOUT_B, 0, S});
  F.push_back({e->tin_w, X, X, X, 0, 1, K_TIN_W, 0, S});
  F.push_back({e->tin_b, 1, X, X, 0, 1, K_TIN_B, 0, S});
  F.push_back({e->tout_w, X, X, X, 0, 1, K_TOUT_W, 0, S});
  F.push_back({e->tout_b, 1, X, X, 0, 1, K_TOUT_B, 0, S});
  for (const Fill& f : F)
    if (!fill(e, seed, f)) return false;
  CK(cudaStreamSynchronize(e->stream));
  return build_mods(e);
}

bool create(pi05_engine* e) {
  const pi05_config& c = e->cfg;
  CK(cudaSetDevice(e->device));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, e->device));
  if (prop.major != 10) return set_err(e, "this engine is built for sm_100a (B200); device is sm_" +
                                              std::to_string(prop.major) + std::to_string(prop.minor));
  e->num_sms = prop.multiProcessorCount;
  // PI05_PDL=0 launches without programmatic dependent launch (each kernel waits for the previous one)
  if (const char* s = getenv("PI05_PDL")) e->pdl = atoi(s) != 0;
  if (const char* s = getenv("PI05_CLUSTER_SPLITK")) e->cluster_splitk = atoi(s) != 0;
  if (const char* s = getenv("PI05_ATTN_TC")) e->attn_tc = atoi(s) != 0;
  if (const char* s = getenv("PI05_ATTN_BWD_PIPE")) e->attn_bwd_pipe = atoi(s) != 0;
  if (const char* s = getenv("PI05_ATTN_WS_HALF")) e->attn_ws_half = atoi(s) != 0;
  if (const char* s = getenv("PI05_WIDE_SWAP")) e->wide_swap = atoi(s) != 0;
  if (const char* s = getenv("PI05_GEMM_WIDE")) e->gemm_wide = atoi(s) != 0;
  if (const char* s = getenv("PI05_GEMM_PAIR")) e->gemm_pair = atoi(s) != 0;
  if (const char* s = getenv("PI05_MEGA")) e->mega = atoi(s) != 0;
  if (const char* s = getenv("PI05_FUSE_NORM")) e->fuse_norm = atoi(s) != 0;
  if (const char* s = getenv("PI05_FUSE_GEGLU_BWD")) e->fuse_geglu_bwd = atoi(s) != 0;
  CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) return set_err(e, "cuTensorMapEncodeTiled unavailable");
  e->encode = reinterpret_cast<EncodeTiledFn>(fn);

  if (!set_gemm_smem<64>(e) || !set_gemm_smem<128>(e) || !set_gemm_smem<256>(e)) return false;
  if (!set_gemm_smem_small<16>(e) || !set_gemm_smem_small<32>(e) || !set_gemm_smem_small<48>(e)) return false;
  if (!set_swap_cluster_smem<64>(e) || !set_swap_cluster_smem<128>(e) || !set_swap_cluster_smem<256>(e)) return false;
  if (!set_gemm_wide_smem(e) || !set_gemm_pair_smem(e)) return false;

  CK(cudaFuncSetAttribute(attn_kernel<P5_HD, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnCfg<P5_HD, 4>::SMEM));
  CK(cudaFuncSetAttribute(attn_kernel<P5_HD, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnCfg<P5_HD, 8>::SMEM));
  CK(cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTcCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_sig_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSigCfg::SMEM));
  CK(cudaFuncSetAttribute(denoise_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MegaCfg::SMEM));
  CK(cudaFuncSetAttribute(attn_kernel<P5_SIG_HD, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnCfg<P5_SIG_HD, 4>::SMEM));
  CK(cudaFuncSetAttribute(attn_kernel<P5_SIG_HD, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnCfg<P5_SIG_HD, 8>::SMEM));

  // weights
  e->warena = nullptr;
  layout_weights(e);
  e->wbytes = e->wused;
  void* p;
  if (!dalloc(e, &p, e->wbytes)) return false;
  e->warena = (char*)p;
  layout_weights(e);

  // activations
  const int B = e->max_batch, P = e->P, H = c.horizon;
  const long Ts = (long)B * c.n_cameras * P5_SIG_TOK, Tp = (long)B * P, Te = (long)B * H;
  Acts& A = e->A;
  auto al = [&](void** dst, size_t bytes) { return dalloc(e, dst, bytes); };
  if (!al((void**)&A.images, (size_t)B * c.n_cameras * P5_IMG * P5_IMG * 3) ||
      !al((void**)&A.tokens, (size_t)B * std::max(1, c.n_text) * 4) ||
      !al((void**)&A.patches, (size_t)Ts * P5_SIG_KPAD * 2) || !al((void**)&A.sx, (size_t)Ts * P5_SIG_W * 2) ||
      !al((void**)&A.sy, (size_t)Ts * P5_SIG_W * 2) || !al((void**)&A.sqkv, (size_t)Ts * P5_SIG_QKV * 2) ||
      !al((void**)&A.so, (size_t)Ts * P5_SIG_W * 2) || !al((void**)&A.sh, (size_t)Ts * P5_SIG_MLP * 2) ||
      !al((void**)&A.px, (size_t)Tp * P5_GEM_W * 2) || !al((void**)&A.ph, (size_t)Tp * P5_GEM_W * 2) ||
      !al((void**)&A.pqkv, (size_t)Tp * P5_QKV * 2) || !al((void**)&A.po, (size_t)Tp * P5_QDIM * 2) ||
      !al((void**)&A.pact, (size_t)Tp * P5_GEM_MLP * 2) ||
      !al((void**)&A.kcache, (size_t)c.gemma_layers * Tp * P5_HD * 2) ||
      !al((void**)&A.vcache, (size_t)c.gemma_layers * Tp * P5_HD * 2) ||
      !al((void**)&A.ex, (size_t)Te * P5_EXP_W * 2) || !al((void**)&A.eh, (size_t)Te * P5_EXP_W * 2) ||
      !al((void**)&A.eqkv, (size_t)Te * P5_QKV * 2) || !al((void**)&A.eo, (size_t)Te * P5_QDIM * 2) ||
      !al((void**)&A.eact, (size_t)Te * P5_EXP_MLP * 2) || !al((void**)&A.ek, (size_t)Te * P5_HD * 2) ||
      !al((void**)&A.ev, (size_t)Te * P5_HD * 2) || !al((void**)&A.xt, (size_t)Te * P5_ACT_D * 4) ||
      !al((void**)&A.noise, (size_t)Te * P5_ACT_D * 4) || !al((void**)&A.actions, (size_t)Te * P5_ACT_D * 4))
    return false;
  // RoPE table, modulation table, GEMM and attention workspaces, status word
  const int npos = P + H + 8;
  std::vector<float> cs((size_t)npos * 128), sn((size_t)npos * 128);
  p5_rope_table(npos, cs.data(), sn.data());
  if (!al((void**)&e->d_cos, cs.size() * 4) || !al((void**)&e->d_sin, sn.size() * 4)) return false;
  CK(cudaMemcpyAsync(e->d_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaMemcpyAsync(e->d_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, e->stream));
  if (!al((void**)&e->mods, (size_t)c.num_steps * e->NM * 3 * P5_EXP_W * 2)) return false;
  e->gemm_ws_bytes = (size_t)64 << 20;
  e->n_counters = 1 << 16;
  if (!al((void**)&e->gemm_ws, e->gemm_ws_bytes) || !al((void**)&e->counters, (size_t)e->n_counters * 4)) return false;
  e->attn_ws_rows = (size_t)4 * 16 * H * P5_NH;
  if (!al((void**)&e->attn_ws_o, e->attn_ws_rows * P5_HD * 4) || !al((void**)&e->attn_ws_ml, e->attn_ws_rows * 2 * 4))
    return false;
  if (!al((void**)&e->d_status, 64)) return false;
  if (!al((void**)&e->d_valid, (size_t)B * sizeof(int))) return false;
  if (!al((void**)&e->nrm_ss, (size_t)2 * (P5_EXP_W / 16) * 64 * 4)) return false;
  CK(cudaStreamSynchronize(e->stream));
  return true;
}

}  // namespace

#include "train.cuh"

// ===================================================================== C ABI
extern "C" {

void pi05_default_config(pi05_config* c) {
  if (!c) return;
  c->batch_invariant = 0;
  c->text_pad_mask = 0;
  c->prefix_group = 0;
  c->siglip_layers = 27;
  c->gemma_layers = 18;
  c->expert_layers = 18;
  c->num_steps = 10;
  c->n_cameras = 3;
  c->n_text = 200;
  c->horizon = 50;
}

pi05_engine* pi05_create(const pi05_config* c, int device, int max_batch, char* err, size_t err_len) {
  auto fail = [&](const std::string& m) -> pi05_engine* {
    if (err && err_len) snprintf(err, err_len, "%s", m.c_str());
    return nullptr;
  };
  pi05_config cfg;
  pi05_default_config(&cfg);
  if (c) cfg = *c;
  if (cfg.siglip_layers < 0 || cfg.gemma_layers < 1 || cfg.expert_layers != cfg.gemma_layers || cfg.num_steps < 1 ||
      cfg.n_cameras < 1 || cfg.n_text < 0 || cfg.horizon < 1 || cfg.horizon > 128 || max_batch < 1 ||
      (cfg.batch_invariant != 0 && cfg.batch_invariant != 1) || (cfg.text_pad_mask != 0 && cfg.text_pad_mask != 1) ||
      cfg.prefix_group < 0 || cfg.prefix_group > cfg.n_cameras * P5_SIG_TOK + cfg.n_text || max_batch > 32767)
    return fail("pi05_create: invalid configuration");
  pi05_engine* e = new pi05_engine();
  e->cfg = cfg;
  e->device = device;
  e->max_batch = max_batch;
  e->P = cfg.n_cameras * P5_SIG_TOK + cfg.n_text;
  e->NM = 2 * cfg.expert_layers + 1;
  if (!create(e)) {
    std::string m = e->err;
    pi05_destroy(e);
    return fail("pi05_create: " + m);
  }
  return e;
}

void pi05_destroy(pi05_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& kv : e->denoise_graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : e->prefill_graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : e->prefill_emb_graphs) cudaGraphExecDestroy(kv.second);
  if (e->tr) dp_release(e->tr->dp);
  delete e->tr;
  for (void* p : e->allocs) cudaFree(p);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

const char* pi05_last_error(const pi05_engine* e) { return e ? e->err.c_str() : "null engine"; }

int pi05_prefix_len(const pi05_engine* e) { return e ? e->P : 0; }

void* pi05_stream(pi05_engine* e) { return e ? (void*)e->stream : nullptr; }

int pi05_sync(pi05_engine* e) {
  if (!e) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  cudaError_t ce = cudaStreamSynchronize(e->stream);
  if (ce != cudaSuccess) {
    e->err = std::string("cudaStreamSynchronize: ") + cudaGetErrorString(ce);
    return PI05_ERR_CUDA;
  }
  if (!check_status(e)) return fail_code(e);
  return PI05_OK;
}

int pi05_init_random_weights(pi05_engine* e, uint64_t seed) {
  if (!e) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  if (!init_random(e, seed)) return fail_code(e);
  e->weights_ready = true;
  ++e->wgen;  // weight-derived copies (the persistent denoise's q/k/v row permutation) are stale
  e->prefix_n = 0;
  return PI05_OK;
}

int pi05_save_weights(pi05_engine* e, const char* path) {
  if (!e || !path) return PI05_ERR_ARG;
  if (!e->weights_ready) {
    e->err = "no weights";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  FILE* f = fopen(path, "wb");
  if (!f) {
    e->err = std::string("cannot open ") + path;
    return PI05_ERR_ARG;
  }
  std::string man = "pi05w 1\n";
  const pi05_config& c = e->cfg;
  man += "cfg siglip_layers " + std::to_string(c.siglip_layers) + "\ncfg gemma_layers " +
         std::to_string(c.gemma_layers) + "\ncfg expert_layers " + std::to_string(c.expert_layers) +
         "\ncfg num_steps " + std::to_string(c.num_steps) + "\ncfg n_cameras " + std::to_string(c.n_cameras) +
         "\ncfg n_text " + std::to_string(c.n_text) + "\ncfg horizon " + std::to_string(c.horizon) + "\n";
  size_t off = 0;
  for (const Tensor& t : e->tensors) {
    const size_t bytes = (size_t)t.rows * t.cols * 2;
    man += "t " + t.name + " bf16 " + std::to_string(off) + " " + std::to_string(bytes) + " " +
           std::to_string(t.rows) + " " + std::to_string(t.cols) + "\n";
    off += (bytes + 255) & ~(size_t)255;
  }
  man += "end\n";
  const size_t hdr = (man.size() + 255) & ~(size_t)255;
  man.resize(hdr, '\n');
  fwrite(man.data(), 1, hdr, f);
  std::vector<char> buf;
  for (const Tensor& t : e->tensors) {
    const size_t bytes = (size_t)t.rows * t.cols * 2, padded = (bytes + 255) & ~(size_t)255;
    buf.assign(padded, 0);
    if (cudaMemcpy(buf.data(), t.ptr, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
      fclose(f);
      e->err = "device read failed";
      return PI05_ERR_CUDA;
    }
    fwrite(buf.data(), 1, padded, f);
  }
  fclose(f);
  return PI05_OK;
}

}  // extern "C"

namespace {

// ------------------------------------------------------------------ weight files (.pi05w)
// A text manifest -- "pi05w <version>", "cfg <key> <value>" lines (the model hyper-parameters),
// "t <name> <bf16|f32> <offset> <bytes> <dims...>" lines, "end" -- padded to 256 bytes, then the raw
// tensors at 256-byte aligned offsets from the end of the manifest (the reference's format,
// π05_네이티브엔진.md:46-47).
struct WEntry {
  size_t off = 0, bytes = 0;
  int f32 = 0;  // element type in the file: bf16 or f32 (f32 is rounded to bf16 on load, as the reference
                // cast its f32 orbax weights, π05_네이티브엔진.md:32)
  long n = 0;   // elements
};

struct WFile {
  FILE* f = nullptr;
  size_t hdr = 0;
  std::map<std::string, long> cfg;
  std::map<std::string, WEntry> ent;
  ~WFile() {
    if (f) fclose(f);
  }
};

bool read_manifest(const char* path, WFile& W, std::string& err) {
  W.f = fopen(path, "rb");
  if (!W.f) {
    err = std::string("cannot open ") + path;
    return false;
  }
  std::vector<std::string> lines;
  std::string cur;
  size_t consumed = 0;
  int ch;
  while ((ch = fgetc(W.f)) != EOF) {
    ++consumed;
    if (ch == '\n') {
      if (cur == "end") break;
      lines.push_back(cur);
      cur.clear();
      if (lines.size() > (1u << 20)) break;
    } else {
      cur.push_back((char)ch);
    }
  }
  W.hdr = (consumed + 255) & ~(size_t)255;
  if (lines.empty() || lines[0].rfind("pi05w", 0) != 0) {
    err = "not a pi05w file";
    return false;
  }
  for (const std::string& L : lines) {
    char name[256], dt[16];
    long v = 0;
    size_t off = 0, bytes = 0;
    if (sscanf(L.c_str(), "cfg %255s %ld", name, &v) == 2) {
      W.cfg[name] = v;
    } else if (sscanf(L.c_str(), "t %255s %15s %zu %zu", name, dt, &off, &bytes) == 4) {
      WEntry e;
      e.off = off;
      e.bytes = bytes;
      e.f32 = strcmp(dt, "f32") == 0;
      if (!e.f32 && strcmp(dt, "bf16") != 0) {
        err = std::string("tensor ") + name + ": unsupported dtype " + dt;
        return false;
      }
      e.n = (long)(bytes / (e.f32 ? 4 : 2));
      W.ent[name] = e;
    }
  }
  return true;
}

uint16_t f32_to_bf16_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// Rows [r0, r0 + nr) of a file tensor seen as [rows][src_cols], columns [0, cols), as bf16 bits into
// dst (row pitch dst_ld elements, row step dst_step rows).
bool read_block(WFile& W, const WEntry& e, long src_cols, long r0, long nr, long cols, uint16_t* dst, long dst_ld,
                long dst_step, std::string& err) {
  const size_t es = e.f32 ? 4 : 2;
  std::vector<char> row((size_t)src_cols * es);
  for (long r = 0; r < nr; ++r) {
    const size_t at = W.hdr + e.off + ((size_t)(r0 + r) * src_cols) * es;
    if (fseek(W.f, (long)at, SEEK_SET) != 0 || fread(row.data(), 1, row.size(), W.f) != row.size()) {
      err = "short read";
      return false;
    }
    uint16_t* d = dst + (size_t)r * dst_step * dst_ld;
    if (e.f32) {
      const float* sf = reinterpret_cast<const float*>(row.data());
      for (long c = 0; c < cols; ++c) d[c] = f32_to_bf16_bits(sf[c]);
    } else {
      memcpy(d, row.data(), (size_t)cols * 2);
    }
  }
  return true;
}

// Assemble the engine tensor `t` from the file: under its own name, or from the reference's layout --
// separate q / k / v and gate / up tensors ([out][in] each; gate/up rows interleaved here), the SigLIP
// MLP padded 4304 -> 4352 (the padding dropped), the patch embedding at 588 columns (padded here to
// 640 with zeros), and one adaRMS modulation Dense per norm.
bool gather_tensor(pi05_engine* e, WFile& W, const Tensor& t, std::vector<uint16_t>& out, std::string& err) {
  const long R = t.rows, C = t.cols;
  out.assign((size_t)R * C, 0);
  auto has = [&](const std::string& n, long elems) {
    auto it = W.ent.find(n);
    return it != W.ent.end() && it->second.n == elems;
  };
  auto rows_of = [&](const std::string& n, long src_cols, long r0, long nr, long cols, long dst_row, long dst_step) {
    return read_block(W, W.ent[n], src_cols, r0, nr, cols, out.data() + (size_t)dst_row * C, C, dst_step, err);
  };
  if (has(t.name, R * C)) return rows_of(t.name, C, 0, R, C, 0, 1);
  const std::string& nm = t.name;
  auto ends = [&](const char* suf) {
    const size_t n = strlen(suf);
    return nm.size() > n && nm.compare(nm.size() - n, n, suf) == 0;
  };
  const std::string stem = nm.substr(0, nm.rfind('.') == std::string::npos ? 0 : nm.rfind('.'));  // "gem.l3.qkv"
  const std::string base = stem.substr(0, stem.rfind('.') + 1);                                    // "gem.l3."
  if (ends(".qkv.w") || ends(".qkv.b")) {
    const bool bias = ends(".b");
    const long D = bias ? 1 : C;
    const bool sig = nm.rfind("sig.", 0) == 0;
    const long fq = sig ? P5_SIG_W : P5_QDIM, fk = sig ? P5_SIG_W : P5_HD;
    const std::string q = base + (bias ? "q.b" : "q.w"), k = base + (bias ? "k.b" : "k.w"), v = base + (bias ? "v.b" : "v.w");
    if (bias) {
      if (has(q, fq) && has(k, fk) && has(v, fk))
        return read_block(W, W.ent[q], fq, 0, 1, fq, out.data(), C, 1, err) &&
               read_block(W, W.ent[k], fk, 0, 1, fk, out.data() + fq, C, 1, err) &&
               read_block(W, W.ent[v], fk, 0, 1, fk, out.data() + fq + fk, C, 1, err);
    } else if (has(q, fq * D) && has(k, fk * D) && has(v, fk * D)) {
      return rows_of(q, D, 0, fq, D, 0, 1) && rows_of(k, D, 0, fk, D, fq, 1) && rows_of(v, D, 0, fk, D, fq + fk, 1);
    }
  } else if (ends(".gu.w")) {
    const long F = R / 2;
    const std::string g = base + "gate.w", u = base + "up.w";
    if (has(g, F * C) && has(u, F * C)) return rows_of(g, C, 0, F, C, 0, 2) && rows_of(u, C, 0, F, C, 1, 2);
  } else if (nm.rfind("sig.", 0) == 0 && (ends(".mlp1.w") || ends(".mlp1.b") || ends(".mlp2.w"))) {
    const long PAD = 4352;  // the reference padded the SigLIP MLP width to a multiple of 128 with zeros
    if (ends(".mlp1.w") && has(nm, PAD * C)) return rows_of(nm, C, 0, R, C, 0, 1);
    if (ends(".mlp1.b") && has(nm, PAD)) return rows_of(nm, PAD, 0, 1, C, 0, 1);
    if (ends(".mlp2.w") && has(nm, R * PAD)) return rows_of(nm, PAD, 0, R, C, 0, 1);
  } else if (nm == "sig.stem.w" && has(nm, R * P5_SIG_K)) {
    return rows_of(nm, P5_SIG_K, 0, R, P5_SIG_K, 0, 1);
  } else if (nm == "exp.ada.w" || nm == "exp.ada.b") {
    const bool bias = nm == "exp.ada.b";
    const long per = 3L * P5_EXP_W;
    for (int m = 0; m < e->NM; ++m) {
      const std::string n = m == e->NM - 1 ? std::string("exp.final.ada") + (bias ? ".b" : ".w")
                                           : "exp.l" + std::to_string(m / 2) + ".ada" + std::to_string(m % 2 + 1) +
                                                 (bias ? ".b" : ".w");
      if (bias ? !has(n, per) : !has(n, per * C)) {
        err = "weight file lacks " + n;
        return false;
      }
      if (!(bias ? read_block(W, W.ent[n], per, 0, 1, per, out.data() + m * per, C, 1, err)
                 : rows_of(n, C, 0, per, C, m * per, 1)))
        return false;
    }
    return true;
  }
  err = "weight file lacks tensor " + nm + " of the configured shape";
  return false;
}

const char* kCfgKeys[] = {"siglip_layers", "gemma_layers", "expert_layers", "num_steps", "n_cameras", "n_text",
                          "horizon"};
int32_t* cfg_field(pi05_config* c, int i) {
  int32_t* f[] = {&c->siglip_layers, &c->gemma_layers, &c->expert_layers, &c->num_steps, &c->n_cameras, &c->n_text,
                  &c->horizon};
  return f[i];
}

}  // namespace

extern "C" {

int pi05_load_weights(pi05_engine* e, const char* path) {
  if (!e || !path) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  WFile W;
  std::string err;
  if (!read_manifest(path, W, err)) {
    e->err = "pi05_load_weights: " + err;
    return PI05_ERR_ARG;
  }
  for (int i = 0; i < 7; ++i) {
    auto it = W.cfg.find(kCfgKeys[i]);
    if (it != W.cfg.end() && it->second != *cfg_field(&e->cfg, i)) {
      e->err = std::string("pi05_load_weights: the file's ") + kCfgKeys[i] + " " + std::to_string(it->second) +
               " differs from the engine's " + std::to_string(*cfg_field(&e->cfg, i));
      return PI05_ERR_ARG;
    }
  }
  std::vector<uint16_t> buf;
  for (const Tensor& t : e->tensors) {
    if (!gather_tensor(e, W, t, buf, err)) {
      e->err = "pi05_load_weights: " + err;
      return PI05_ERR_ARG;
    }
    if (cudaMemcpy(t.ptr, buf.data(), buf.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
      e->err = "device write failed";
      return PI05_ERR_CUDA;
    }
  }
  if (!build_mods(e)) return fail_code(e);
  e->weights_ready = true;
  ++e->wgen;  // weight-derived copies (the interleaved q/k/v rows of the fused-RoPE projections) are stale
  e->prefix_n = 0;
  return PI05_OK;
}

int pi05_read_weights_config(const char* path, pi05_config* c) {
  if (!path || !c) return PI05_ERR_ARG;
  WFile W;
  std::string err;
  if (!read_manifest(path, W, err)) return PI05_ERR_ARG;
  pi05_default_config(c);
  for (int i = 0; i < 7; ++i) {
    auto it = W.cfg.find(kCfgKeys[i]);
    if (it != W.cfg.end()) *cfg_field(c, i) = (int32_t)it->second;
  }
  return PI05_OK;
}

int pi05_prefill(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens) {
  if (!e || n < 1 || n > e->max_batch || !images || (e->cfg.n_text > 0 && !tokens)) {
    if (e) e->err = "pi05_prefill: bad arguments";
    return PI05_ERR_ARG;
  }
  if (!e->weights_ready) {
    e->err = "pi05_prefill: weights not loaded";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  const size_t ib = (size_t)n * e->cfg.n_cameras * P5_IMG * P5_IMG * 3;
  if (!copy_in(e, e->A.images, images, ib)) return PI05_ERR_CUDA;
  if (e->cfg.n_text > 0 && !copy_in(e, e->A.tokens, tokens, (size_t)n * e->cfg.n_text * 4)) return PI05_ERR_CUDA;
  if (!prefill_resident(e, n)) return fail_code(e);
  e->prefix_n = n;
  return PI05_OK;
}

int pi05_prefill_embeds(pi05_engine* e, int n, const uint8_t* images, const uint16_t* text_emb) {
  if (!e || n < 1 || n > e->max_batch || !images || (e->cfg.n_text > 0 && !text_emb)) {
    if (e) e->err = "pi05_prefill_embeds: bad arguments";
    return PI05_ERR_ARG;
  }
  if (e->cfg.text_pad_mask) {
    e->err = "pi05_prefill_embeds: the prompt padding mask reads token ids (text_pad_mask must be 0)";
    return PI05_ERR_ARG;
  }
  if (!e->weights_ready) {
    e->err = "pi05_prefill_embeds: weights not loaded";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  const size_t tb = (size_t)e->cfg.n_text * P5_GEM_W * 2;  // one sample's text rows
  if (tb > 0 && !e->text_emb && !dalloc(e, (void**)&e->text_emb, (size_t)e->max_batch * tb)) return PI05_ERR_CUDA;
  const size_t ib = (size_t)n * e->cfg.n_cameras * P5_IMG * P5_IMG * 3;
  if (!copy_in(e, e->A.images, images, ib)) return PI05_ERR_CUDA;
  if (tb > 0 && !copy_in(e, e->text_emb, text_emb, (size_t)n * tb)) return PI05_ERR_CUDA;
  e->text_from_emb = true;
  const bool ok = prefill_resident(e, n);
  e->text_from_emb = false;
  if (!ok) return fail_code(e);
  e->prefix_n = n;
  return PI05_OK;
}

int pi05_set_prefix_cache(pi05_engine* e, int n, const uint16_t* k, const uint16_t* v) {
  if (!e || n < 1 || n > e->max_batch || !k || !v) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  const size_t per = (size_t)e->P * P5_HD;  // one layer of one sample
  const size_t layer = (size_t)e->max_batch * per;
  for (int l = 0; l < e->cfg.gemma_layers; ++l)
    for (int b = 0; b < n; ++b) {
      const size_t src = ((size_t)b * e->cfg.gemma_layers + l) * per;
      if (!copy_in(e, e->A.kcache + l * layer + b * per, k + src, per * 2) ||
          !copy_in(e, e->A.vcache + l * layer + b * per, v + src, per * 2))
        return PI05_ERR_CUDA;
    }
  if (!is_device_ptr(k) && cudaStreamSynchronize(e->stream) != cudaSuccess) return PI05_ERR_CUDA;
  if (!set_valid_full(e, n)) return PI05_ERR_CUDA;
  e->prefix_n = n;
  return PI05_OK;
}

int pi05_synth_prefix_cache(pi05_engine* e, int n, uint64_t seed) {
  if (!e || n < 1 || n > e->max_batch) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  const size_t per = (size_t)e->P * P5_HD;
  const size_t layer = (size_t)e->max_batch * per;
  const float sc = p5_scale_for_std(1.0);
  for (int b = 0; b < n; ++b) {
    // stream per sample, logical index (l * P + p) * 256 + d, as the host generator lays it out
    const uint64_t kk = p5_key(seed, K_IN_KCACHE, (uint32_t)b), kv = p5_key(seed, K_IN_VCACHE, (uint32_t)b);
    for (int l = 0; l < e->cfg.gemma_layers; ++l) {
      // generate the [P][256] block of layer l: logical offset l*per
      fill_normal_bf16_kernel<<<148, 256, 0, e->stream>>>(e->A.kcache + l * layer + b * per, (long)per, kk, sc,
                                                          (long)(l * per));
      fill_normal_bf16_kernel<<<148, 256, 0, e->stream>>>(e->A.vcache + l * layer + b * per, (long)per, kv, sc,
                                                          (long)(l * per));
    }
  }
  if (!set_valid_full(e, n)) return PI05_ERR_CUDA;
  e->prefix_n = n;
  return cudaGetLastError() == cudaSuccess ? PI05_OK : PI05_ERR_CUDA;
}

int pi05_get_prefix_cache(pi05_engine* e, int sample, int layer, uint16_t* k, uint16_t* v) {
  if (!e || sample < 0 || sample >= e->max_batch || layer < 0 || layer >= e->cfg.gemma_layers) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  const size_t per = (size_t)e->P * P5_HD;
  const size_t off = (size_t)layer * e->max_batch * per + (size_t)sample * per;
  if (cudaMemcpyAsync(k, e->A.kcache + off, per * 2, cudaMemcpyDefault, e->stream) != cudaSuccess ||
      cudaMemcpyAsync(v, e->A.vcache + off, per * 2, cudaMemcpyDefault, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  return pi05_sync(e);
}

int pi05_denoise(pi05_engine* e, int n, const float* noise, float* actions) {
  if (!e || n < 1 || n > e->max_batch || !noise || !actions) return PI05_ERR_ARG;
  if (!e->weights_ready || e->prefix_n < n) {
    e->err = "pi05_denoise: no prefix cache for this batch (call pi05_prefill first)";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  const size_t bytes = (size_t)n * e->cfg.horizon * P5_ACT_D * 4;
  if (!copy_in(e, e->A.xt, noise, bytes)) return PI05_ERR_CUDA;
  if (!denoise_resident(e, n)) return fail_code(e);
  if (cudaMemcpyAsync(actions, e->A.xt, bytes, cudaMemcpyDefault, e->stream) != cudaSuccess) return PI05_ERR_CUDA;
  if (!is_device_ptr(actions)) return pi05_sync(e);
  return PI05_OK;
}

int pi05_infer(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* noise,
               float* actions) {
  int rc = pi05_prefill(e, n, images, tokens);
  if (rc != PI05_OK) return rc;
  return pi05_denoise(e, n, noise, actions);
}

}  // extern "C"

namespace {

int verify_run(pi05_engine* e, const uint8_t* images, const int32_t* tokens, const float* noise, float* actions,
               pi05_probe_fn probe, pi05_plant_fn plant, void* ctx) {
  if (!e) return PI05_ERR_ARG;
  if (!images || (e->cfg.n_text > 0 && !tokens) || !noise) {
    e->err = "pi05_verify: bad arguments";
    return PI05_ERR_ARG;
  }
  if (!e->weights_ready) {
    e->err = "pi05_verify: weights not loaded";
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  const size_t ib = (size_t)e->cfg.n_cameras * P5_IMG * P5_IMG * 3, ab = (size_t)e->cfg.horizon * P5_ACT_D * 4;
  if (!copy_in(e, e->A.images, images, ib)) return PI05_ERR_CUDA;
  if (e->cfg.n_text > 0 && !copy_in(e, e->A.tokens, tokens, (size_t)e->cfg.n_text * 4)) return PI05_ERR_CUDA;
  if (!copy_in(e, e->A.xt, noise, ab)) return PI05_ERR_CUDA;
  if (!qkv_interleave_prepare(e)) return fail_code(e);
  e->probe_fn = probe;
  e->plant_fn = plant;
  e->probe_ctx = ctx;
  bool ok = run_prefill_body(e, 1);
  if (ok) e->prefix_n = 1;
  ok = ok && run_denoise_body(e, 1);
  e->probe_fn = nullptr;
  e->plant_fn = nullptr;
  e->probe_ctx = nullptr;
  if (!ok) return fail_code(e);
  if (actions && cudaMemcpyAsync(actions, e->A.xt, ab, cudaMemcpyDefault, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  return pi05_sync(e);
}

}  // namespace

extern "C" {

int pi05_verify(pi05_engine* e, const uint8_t* images, const int32_t* tokens, const float* noise, float* actions,
                pi05_probe_fn fn, void* ctx) {
  return verify_run(e, images, tokens, noise, actions, fn, nullptr, ctx);
}

int pi05_verify_planted(pi05_engine* e, const uint8_t* images, const int32_t* tokens, const float* noise,
                        float* actions, pi05_plant_fn fn, void* ctx) {
  if (!fn) return PI05_ERR_ARG;
  return verify_run(e, images, tokens, noise, actions, nullptr, fn, ctx);
}

// kernels per call, as captured (for launch accounting in benchmarks)
long pi05_graph_launches(pi05_engine* e, int which, int n) {
  if (!e) return -1;
  auto& m = which == 0 ? e->prefill_launches : e->denoise_launches;
  auto it = m.find(n);
  return it == m.end() ? -1 : it->second;
}

void pi05_synth_images(uint64_t seed, int sample, int n_cameras, uint8_t* out) {
  const uint64_t key = p5_key(seed, K_IN_IMAGE, (uint32_t)sample);
  const long n = (long)n_cameras * P5_IMG * P5_IMG * 3;
  for (long i = 0; i < n; ++i) out[i] = p5_u8(key, (uint64_t)i);
}
void pi05_synth_tokens(uint64_t seed, int sample, int n_text, int32_t* out) {
  const uint64_t key = p5_key(seed, K_IN_TOKENS, (uint32_t)sample);
  for (int i = 0; i < n_text; ++i) out[i] = p5_token(key, (uint64_t)i);
}
void pi05_synth_noise(uint64_t seed, int sample, int horizon, float* out) {
  const uint64_t key = p5_key(seed, K_IN_NOISE, (uint32_t)sample);
  const float sc = p5_scale_for_std(1.0);
  for (long i = 0; i < (long)horizon * P5_ACT_D; ++i) out[i] = p5_normal(key, (uint64_t)i, sc);
}

int pi05_op_linear(pi05_engine* e, int T, int F, int K, const void* x, const void* w, const void* bias,
                   const void* res, const void* gate, int epi, void* out) {
  if (!e) return PI05_ERR_ARG;
  if (T < 1 || F < 1 || K < 8 || K % 8 || epi < EPI_STORE || epi > EPI_F32 || !x || !w || !out ||
      ((epi == EPI_RESID || epi == EPI_GATED) && !res) || (epi == EPI_GATED && !gate) || (epi == EPI_GEGLU && F % 32)) {
    set_err(e, "pi05_op_linear: bad shape or missing operand (K % 8 == 0, GeGLU F % 32 == 0, res/gate for epi 2/3)");
    return PI05_ERR_ARG;
  }
  // the normal-orientation epilogue moves 8 bf16 (or 4 fp32) values per access: rows of out, res and the
  // bias/gate vectors must start on 16-byte boundaries
  const uintptr_t al = (uintptr_t)x | (uintptr_t)w | (uintptr_t)out | (uintptr_t)bias | (uintptr_t)res | (uintptr_t)gate;
  if (F % 8 || (al & 15)) {
    set_err(e, "pi05_op_linear: F must be a multiple of 8 and x, w, out, bias, res, gate 16-byte aligned");
    return PI05_ERR_ARG;
  }
  cudaSetDevice(e->device);
  Lin L{(const bf16*)x, K, T, (const bf16*)w, K, F, K};
  L.epi = epi;
  const int fo = epi == EPI_GEGLU ? F / 2 : F;
  if (epi == EPI_F32) {
    L.out_f32 = (float*)out;
    L.ld_out_f32 = F;
  } else {
    L.out = (bf16*)out;
    L.ld_out = fo;
  }
  L.bias = (const bf16*)bias;
  L.res = (const bf16*)res;
  L.ld_res = F;
  L.gate = (const bf16*)gate;
  L.ld_gate = 0;
  L.gate_div = 1;
  if (!linear(e, L)) return fail_code(e);
  return PI05_OK;
}

// Device time of one linear layer: `reps` launches captured in a CUDA graph, each on its own copy of the
// weights (enough copies to exceed 256 MB, so every launch streams its weights from HBM, not L2).
int pi05_op_bench_linear(pi05_engine* e, int T, int F, int K, int epi, int reps, float* us_per_launch) {
  if (!e || T < 1 || F < 1 || K < 64 || K % 8 || reps < 1 || !us_per_launch || epi < EPI_STORE || epi > EPI_F32 ||
      (epi == EPI_GEGLU && F % 32))
    return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  const size_t wbytes = (size_t)F * K * 2;
  const int copies = (int)std::max<size_t>(1, std::min<size_t>(64, ((256ull << 20) + wbytes - 1) / wbytes));
  std::vector<void*> bufs;
  auto release = [&]() {
    cudaStreamSynchronize(e->stream);
    for (void* p : bufs) cudaFree(p);
  };
  void *x = nullptr, *out = nullptr, *res = nullptr, *gate = nullptr;
  if (cudaMalloc(&x, (size_t)T * K * 2) != cudaSuccess) return PI05_ERR_CUDA;
  bufs.push_back(x);
  if (cudaMalloc(&out, (size_t)T * F * 4) != cudaSuccess || cudaMalloc(&res, (size_t)T * F * 2) != cudaSuccess ||
      cudaMalloc(&gate, (size_t)F * 2) != cudaSuccess) {
    release();
    return PI05_ERR_CUDA;
  }
  bufs.push_back(out);
  bufs.push_back(res);
  bufs.push_back(gate);
  std::vector<bf16*> ws;
  for (int c = 0; c < copies; ++c) {
    void* w = nullptr;
    if (cudaMalloc(&w, wbytes) != cudaSuccess) {
      release();
      return PI05_ERR_CUDA;
    }
    bufs.push_back(w);
    ws.push_back((bf16*)w);
    fill_param_kernel<<<148 * 4, 256, 0, e->stream>>>((bf16*)w, F, K, K, 0, 1, p5_key(c, 999, 0),
                                                     p5_scale_for_std(0.02), 0.f);
  }
  fill_param_kernel<<<148 * 4, 256, 0, e->stream>>>((bf16*)x, T, K, K, 0, 1, p5_key(1, 998, 0), p5_scale_for_std(1.0),
                                                   0.f);
  cudaMemsetAsync(res, 0, (size_t)T * F * 2, e->stream);
  cudaMemsetAsync(gate, 0, (size_t)F * 2, e->stream);
  auto one = [&](int i) {
    Lin L{(const bf16*)x, K, T, ws[i % copies], K, F, K};
    L.epi = epi;
    if (epi == EPI_F32) {
      L.out_f32 = (float*)out;
      L.ld_out_f32 = F;
    } else {
      L.out = (bf16*)out;
      L.ld_out = epi == EPI_GEGLU ? F / 2 : F;
    }
    L.res = (const bf16*)res;
    L.ld_res = F;
    L.gate = (const bf16*)gate;
    return linear(e, L);
  };
  // warm-up (also sets up every launch's tensor maps), then capture and replay
  for (int i = 0; i < std::min(reps, copies); ++i)
    if (!one(i)) {
      release();
      return fail_code(e);
    }
  cudaGraph_t g = nullptr;
  cudaGraphExec_t gx = nullptr;
  if (cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    release();
    return PI05_ERR_CUDA;
  }
  bool ok = true;
  for (int i = 0; i < reps && ok; ++i) ok = one(i);
  cudaStreamEndCapture(e->stream, &g);
  if (!ok || !g || cudaGraphInstantiate(&gx, g, 0) != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    release();
    return ok ? PI05_ERR_CUDA : fail_code(e);
  }
  cudaGraphDestroy(g);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaGraphLaunch(gx, e->stream);  // warm replay
  cudaEventRecord(e0, e->stream);
  cudaGraphLaunch(gx, e->stream);
  cudaEventRecord(e1, e->stream);
  cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  *us_per_launch = ms * 1000.0f / reps;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(gx);
  release();
  return check_status(e) ? PI05_OK : fail_code(e);
}

int pi05_op_attention(pi05_engine* e, int batch, int T, int S, const void* q, int ldq, const void* k, const void* v,
                      void* out, int splits) {
  if (!e || batch < 1 || T < 1 || S < 1 || ldq < P5_QDIM || ldq % 8 || !q || !k || !v || !out || splits < 0)
    return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  AttnArgs at = {};
  at.q = (const bf16*)q;
  at.ldq = ldq;
  at.q_bstride = (long)T * ldq;
  at.out = (bf16*)out;
  at.ldo = P5_QDIM;
  at.o_bstride = (long)T * P5_QDIM;
  at.k1 = (const bf16*)k;
  at.v1 = (const bf16*)v;
  at.ld1 = P5_HD;
  at.len1 = S;
  at.b1stride = (long)S * P5_HD;
  at.k2 = at.k1;
  at.v2 = at.v1;
  at.T = T;
  at.G = P5_NH;
  at.qdiv = 1.0f;
  at.splits = splits > 0 ? splits : 8;
  at.force_splits = splits;  // 0: chosen by the engine
  if (!attention(e, at, batch, P5_HD)) return fail_code(e);
  return PI05_OK;
}

int pi05_op_siglip_attention(pi05_engine* e, int images, const void* qkv, void* out) {
  if (!e || images < 1 || images > 65535 || !qkv || !out) return PI05_ERR_ARG;
  cudaSetDevice(e->device);
  AttnArgs at = {};
  at.q = (const bf16*)qkv;
  at.ldq = P5_SIG_QKV;
  at.q_bstride = (long)P5_SIG_TOK * P5_SIG_QKV;
  at.out = (bf16*)out;
  at.ldo = P5_SIG_W;
  at.o_bstride = (long)P5_SIG_TOK * P5_SIG_W;
  at.k1 = (const bf16*)qkv + P5_SIG_W;
  at.v1 = (const bf16*)qkv + 2 * P5_SIG_W;
  at.ld1 = P5_SIG_QKV;
  at.len1 = P5_SIG_TOK;
  at.b1stride = (long)P5_SIG_TOK * P5_SIG_QKV;
  at.k2 = at.k1;
  at.v2 = at.v1;
  at.T = P5_SIG_TOK;
  at.G = 1;
  at.qdiv = P5_SIG_QDIV;
  at.splits = 1;
  if (!attention(e, at, images, P5_SIG_HD)) return fail_code(e);
  return PI05_OK;
}

pi05_engine* pi05_create_batch(const char* weights_path, int device, int max_batch) {
  char err[512];
  pi05_config cfg;
  if (weights_path ? pi05_read_weights_config(weights_path, &cfg) != PI05_OK : false) return nullptr;
  pi05_engine* e = pi05_create(weights_path ? &cfg : nullptr, device, max_batch, err, sizeof(err));
  if (!e) return nullptr;
  const int rc = weights_path ? pi05_load_weights(e, weights_path) : pi05_init_random_weights(e, 0);
  if (rc != PI05_OK) {
    pi05_destroy(e);
    return nullptr;
  }
  return e;
}

int pi05_infer_batch(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* noise,
                     float* actions) {
  return pi05_infer(e, n, images, tokens, noise, actions);
}

int pi05_set_stage(pi05_engine* e, int slot, int stage, int mode) {
  if (!e || slot < 0 || slot >= e->max_batch || stage < 0 || mode < 0 || mode > 1) return PI05_ERR_ARG;
  return PI05_OK;
}

// Receding-horizon stepping over environment slots (reference pi05_act_batch, π05_네이티브엔진.md:292-297
// and :33: camera frames as the evaluator passes them, the chunk re-planned after a fixed number of
// executed steps, actions returned as the wrapper returns them).
int pi05_set_act_config(pi05_engine* e, const pi05_act_config* c) {
  if (!e || !c) return PI05_ERR_ARG;
  if (c->act_dim < 1 || c->act_dim > P5_ACT_D || c->replan < 1 || c->replan > e->cfg.horizon ||
      (!c->mean) != (!c->std)) {
    set_err(e, "pi05_set_act_config: needs 1 <= act_dim <= 32, 1 <= replan <= horizon, mean and std both or neither");
    return PI05_ERR_ARG;
  }
  e->act_dim = c->act_dim;
  e->act_replan = c->replan;
  e->act_mean.clear();
  e->act_std.clear();
  e->act_delta.clear();
  if (c->mean) {
    e->act_mean.assign(c->mean, c->mean + c->act_dim);
    e->act_std.assign(c->std, c->std + c->act_dim);
  }
  if (c->delta_mask) e->act_delta.assign(c->delta_mask, c->delta_mask + c->act_dim);
  e->act_seed = c->noise_seed;
  e->act_chunk.assign(e->max_batch, std::vector<float>());
  e->act_next.assign(e->max_batch, 0);
  e->act_plans.assign(e->max_batch, 0);
  return PI05_OK;
}

namespace {

// Resize the camera frames of the m re-planning slots into batch positions [0, m) of A.images.
bool stage_frames(pi05_engine* e, const std::vector<const pi05_frame*>& fr) {
  const int ncam = e->cfg.n_cameras, m = (int)fr.size() / ncam;
  std::vector<p5rs::FrameJob> jobs(fr.size());
  std::vector<int32_t> tab;
  size_t host_bytes = 0;
  std::vector<char> on_dev(fr.size(), 0);
  for (size_t j = 0; j < fr.size(); ++j) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, fr[j]->data) != cudaSuccess) {
      cudaGetLastError();
      at.type = cudaMemoryTypeUnregistered;
    }
    on_dev[j] = at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
    if (on_dev[j] && at.device != e->device) return set_err(e, "pi05_act_batch: a frame is on another device");
    if (!on_dev[j]) host_bytes += (size_t)fr[j]->height * fr[j]->width * fr[j]->channels;
  }
  void* stage = e->frame_stage;
  if (!grow(e, &stage, &e->frame_stage_bytes, std::max<size_t>(host_bytes, 1))) return false;
  e->frame_stage = (uint8_t*)stage;
  size_t off = 0;
  for (size_t j = 0; j < fr.size(); ++j) {
    const pi05_frame& f = *fr[j];
    p5rs::Geometry g;
    if (!p5rs::geometry(f.height, f.width, P5_IMG, P5_IMG, &g)) return set_err(e, "pi05_act_batch: frame too small to resize");
    p5rs::FrameJob& J = jobs[j];
    J.h = f.height;
    J.w = f.width;
    J.ch = f.channels;
    J.rh = g.rh;
    J.rw = g.rw;
    J.pad_h = g.pad_h;
    J.pad_w = g.pad_w;
    J.dst = e->A.images + j * (size_t)P5_IMG * P5_IMG * 3;  // position j / ncam, camera j % ncam
    if (on_dev[j]) {
      J.src = (const uint8_t*)f.data;
      J.stride = (long)f.stride;
    } else {
      const size_t pitch = (size_t)f.width * f.channels;
      CK(cudaMemcpy2DAsync(e->frame_stage + off, pitch, f.data, (size_t)f.stride, pitch, f.height,
                           cudaMemcpyHostToDevice, e->stream));
      J.src = e->frame_stage + off;
      J.stride = (long)pitch;
      off += pitch * f.height;
    }
    auto add = [&](int n_in, int n_out, int* taps) -> long {
      if (n_in == n_out) return -1;
      const p5rs::AxisTaps t = p5rs::axis_taps(n_in, n_out);
      const long at = (long)tab.size();
      tab.insert(tab.end(), t.first.begin(), t.first.end());
      tab.insert(tab.end(), t.count.begin(), t.count.end());
      tab.insert(tab.end(), t.w.begin(), t.w.end());
      *taps = t.taps;
      return at;
    };
    J.tw = J.th = 0;
    J.tab_w = add(f.width, g.rw, &J.tw);
    J.tab_h = add(f.height, g.rh, &J.th);
  }
  void* tp = e->rs_tab;
  void* jp = e->rs_jobs;
  if (!grow(e, &tp, &e->rs_tab_bytes, std::max<size_t>(tab.size() * 4, 4)) ||
      !grow(e, &jp, &e->rs_jobs_bytes, jobs.size() * sizeof(p5rs::FrameJob)))
    return false;
  e->rs_tab = (int32_t*)tp;
  e->rs_jobs = (p5rs::FrameJob*)jp;
  if (!tab.empty()) CK(cudaMemcpyAsync(e->rs_tab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaMemcpyAsync(e->rs_jobs, jobs.data(), jobs.size() * sizeof(p5rs::FrameJob), cudaMemcpyHostToDevice,
                     e->stream));
  const int px = P5_IMG * P5_IMG;
  resize_with_pad_kernel<<<dim3((px + 255) / 256, (unsigned)jobs.size()), 256, 0, e->stream>>>(e->rs_jobs, e->rs_tab,
                                                                                               P5_IMG, P5_IMG);
  CK(cudaGetLastError());
  (void)m;
  return true;
}

}  // namespace

int pi05_act_batch(pi05_engine* e, int n, const int* slots, const pi05_frame* frames, const int32_t* tokens,
                   const float* state, const float* noise, float* out) {
  if (!e) return PI05_ERR_ARG;
  if (n < 1 || n > e->max_batch || !slots || !frames || (e->cfg.n_text > 0 && !tokens) || !out) {
    set_err(e, "pi05_act_batch: bad arguments");
    return PI05_ERR_ARG;
  }
  if (!e->weights_ready) {
    set_err(e, "pi05_act_batch: weights not loaded");
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  if ((int)e->act_chunk.size() != e->max_batch) {
    e->act_chunk.assign(e->max_batch, std::vector<float>());
    e->act_next.assign(e->max_batch, 0);
    e->act_plans.assign(e->max_batch, 0);
  }
  const int H = e->cfg.horizon, ncam = e->cfg.n_cameras, ad = e->act_dim;
  std::vector<int> need;  // positions in the call whose slot re-plans
  for (int i = 0; i < n; ++i) {
    const int sl = slots[i];
    if (sl < 0 || sl >= e->max_batch) {
      set_err(e, "pi05_act_batch: slot out of range");
      return PI05_ERR_ARG;
    }
    for (int j = 0; j < i; ++j)
      if (slots[j] == sl) {
        set_err(e, "pi05_act_batch: a slot steps at most once per call");
        return PI05_ERR_ARG;
      }
    if (e->act_chunk[sl].empty() || e->act_next[sl] >= e->act_replan) need.push_back(i);
  }
  // state rows (host copy; the dims of the delta mask are added to the re-planned chunks)
  std::vector<float> st;
  if (state && !e->act_delta.empty()) {
    st.resize((size_t)n * ad);
    if (cudaMemcpy(st.data(), state, st.size() * 4, cudaMemcpyDefault) != cudaSuccess) return PI05_ERR_CUDA;
  }
  if (!need.empty()) {
    const int m = (int)need.size();
    std::vector<const pi05_frame*> fr;
    for (int k = 0; k < m; ++k)
      for (int c = 0; c < ncam; ++c) {
        const pi05_frame* f = &frames[(size_t)need[k] * ncam + c];
        if (!f->data || f->height < 1 || f->width < 1 || (f->channels != 3 && f->channels != 4) ||
            f->stride < (int64_t)f->width * f->channels) {
          set_err(e, "pi05_act_batch: bad camera frame (data, height, width, channels 3/4, stride >= width*channels)");
          return PI05_ERR_ARG;
        }
        fr.push_back(f);
      }
    if (!stage_frames(e, fr)) return fail_code(e);
    const size_t nz = (size_t)H * P5_ACT_D;
    for (int k = 0; k < m; ++k) {
      const int i = need[k], sl = slots[i];
      if (e->cfg.n_text > 0 &&
          !copy_in(e, e->A.tokens + (size_t)k * e->cfg.n_text, tokens + (size_t)i * e->cfg.n_text, e->cfg.n_text * 4))
        return PI05_ERR_CUDA;
      if (noise) {
        if (!copy_in(e, e->A.xt + k * nz, noise + i * nz, nz * 4)) return PI05_ERR_CUDA;
      } else {
        // the slot's own stream: plan p of slot s draws elements [p * nz, (p + 1) * nz) of the generator
        // stream (act seed, noise, s); the first plan equals pi05_synth_noise(seed, s)
        std::vector<float> z(nz);
        const uint64_t key = p5_key(e->act_seed, K_IN_NOISE, (uint32_t)sl);
        const float sc = p5_scale_for_std(1.0);
        for (size_t q = 0; q < nz; ++q) z[q] = p5_normal(key, (uint64_t)(e->act_plans[sl] * nz + q), sc);
        float* dst = (e->noise_chol ? e->A.noise : e->A.xt) + k * nz;
        if (cudaMemcpy(dst, z.data(), nz * 4, cudaMemcpyHostToDevice) != cudaSuccess) return PI05_ERR_CUDA;
      }
    }
    if (!noise && e->noise_chol) {  // correlated noise L . eps for every re-planning slot
      const long warps = (long)m * nz;
      correlate_noise_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, e->stream>>>(e->noise_chol, e->A.noise,
                                                                                        e->A.xt, m, (int)nz);
      if (cudaGetLastError() != cudaSuccess) return PI05_ERR_CUDA;
    }
    if (!prefill_resident(e, m)) return fail_code(e);
    e->prefix_n = m;
    if (!denoise_resident(e, m)) return fail_code(e);
    std::vector<float> ch((size_t)m * nz);
    if (cudaMemcpyAsync(ch.data(), e->A.xt, ch.size() * 4, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
      return PI05_ERR_CUDA;
    const int rc = pi05_sync(e);
    if (rc != PI05_OK) return rc;
    // post-process each new chunk as the wrapper does: un-normalise (openpi Unnormalize, z-score), then
    // add the state to the delta dims (AbsoluteActions), keep the first act_dim dims
    const float eps = 1e-6f;
    for (int k = 0; k < m; ++k) {
      const int i = need[k], sl = slots[i];
      std::vector<float>& c = e->act_chunk[sl];
      c.assign((size_t)H * ad, 0.f);
      for (int r = 0; r < H; ++r)
        for (int j = 0; j < ad; ++j) {
          float a = ch[(size_t)k * nz + (size_t)r * P5_ACT_D + j];
          if (!e->act_mean.empty()) a = a * (e->act_std[j] + eps) + e->act_mean[j];
          if (!st.empty() && e->act_delta[j]) a += st[(size_t)i * ad + j];
          c[(size_t)r * ad + j] = a;
        }
      e->act_next[sl] = 0;
      ++e->act_plans[sl];
    }
  }
  std::vector<float> rows((size_t)n * ad);
  for (int i = 0; i < n; ++i) {
    const int sl = slots[i];
    memcpy(rows.data() + (size_t)i * ad, e->act_chunk[sl].data() + (size_t)e->act_next[sl] * ad, ad * sizeof(float));
    ++e->act_next[sl];
  }
  if (cudaMemcpy(out, rows.data(), rows.size() * 4, cudaMemcpyDefault) != cudaSuccess) return PI05_ERR_CUDA;
  return PI05_OK;
}

int pi05_set_noise_cholesky(pi05_engine* e, const float* L, int dim) {
  if (!e) return PI05_ERR_ARG;
  const int nz = e->cfg.horizon * P5_ACT_D;
  if (!L) {
    if (e->noise_chol) {
      cudaSetDevice(e->device);
      cudaStreamSynchronize(e->stream);
      cudaFree(e->noise_chol);
      e->allocs.erase(std::find(e->allocs.begin(), e->allocs.end(), (void*)e->noise_chol));
      e->noise_chol = nullptr;
    }
    return PI05_OK;
  }
  if (dim != nz) {
    set_err(e, "pi05_set_noise_cholesky: dim must be horizon * 32");
    return PI05_ERR_ARG;
  }
  cudaSetDevice(e->device);
  if (!e->noise_chol && !dalloc(e, (void**)&e->noise_chol, (size_t)nz * nz * 4)) return PI05_ERR_CUDA;
  if (cudaMemcpyAsync(e->noise_chol, L, (size_t)nz * nz * 4, cudaMemcpyDefault, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  return pi05_sync(e);
}

int pi05_set_inpaint(pi05_engine* e, int fixed, float t_min, const float* corr) {
  if (!e) return PI05_ERR_ARG;
  const int H = e->cfg.horizon;
  if (fixed < 0 || fixed >= H || fixed * P5_ACT_D * 4 > 48 * 1024 || (fixed > 0 && !corr) || !(t_min == t_min)) {
    set_err(e, "pi05_set_inpaint: fixed must be in [0, horizon) and at most 384 rows, corr given when fixed > 0");
    return PI05_ERR_ARG;
  }
  cudaSetDevice(e->device);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) return PI05_ERR_CUDA;
  // the denoise graphs hold the inpainting launches (or their absence): capture them again
  for (auto& kv : e->denoise_graphs) cudaGraphExecDestroy(kv.second);
  e->denoise_graphs.clear();
  e->denoise_launches.clear();
  auto drop = [&](void* p) {
    if (!p) return;
    cudaFree(p);
    e->allocs.erase(std::find(e->allocs.begin(), e->allocs.end(), p));
  };
  drop(e->inp_corr);
  e->inp_corr = nullptr;
  e->inp_fixed = 0;
  if (fixed == 0) return PI05_OK;
  const int K = fixed * P5_ACT_D, U = H * P5_ACT_D - K;
  const size_t nz = (size_t)e->max_batch * H * P5_ACT_D;
  if (!dalloc(e, (void**)&e->inp_corr, (size_t)U * K * 4)) return PI05_ERR_CUDA;
  // the known rows and the per-position switches keep their size for the engine's life (K <= horizon*32)
  if (!e->inp_known && !dalloc(e, (void**)&e->inp_known, nz * 4)) return PI05_ERR_CUDA;
  if (!e->inp_eps && !dalloc(e, (void**)&e->inp_eps, nz * 4)) return PI05_ERR_CUDA;
  if (!e->inp_on && !dalloc(e, (void**)&e->inp_on, (size_t)e->max_batch * sizeof(int))) return PI05_ERR_CUDA;
  if (cudaMemsetAsync(e->inp_on, 0, (size_t)e->max_batch * sizeof(int), e->stream) != cudaSuccess ||
      cudaMemcpyAsync(e->inp_corr, corr, (size_t)U * K * 4, cudaMemcpyDefault, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  e->inp_fixed = fixed;
  e->inp_tmin = t_min;
  return pi05_sync(e);
}

int pi05_set_kv_mix(pi05_engine* e, const float* wk, const float* bk, const float* wv, const float* bv) {
  if (!e) return PI05_ERR_ARG;
  const int L = e->cfg.gemma_layers;
  if (wk && (!bk || !wv || !bv)) {
    set_err(e, "pi05_set_kv_mix: wk, bk, wv and bv are given together");
    return PI05_ERR_ARG;
  }
  if (wk && L > P5_KV_MIX_MAX_LAYERS) {
    set_err(e, "pi05_set_kv_mix: at most 18 layers");
    return PI05_ERR_ARG;
  }
  if (wk && e->tr) {
    set_err(e, "pi05_set_kv_mix: the LoRA step trains without KV layer mixing");
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) return PI05_ERR_CUDA;
  // the denoise graphs hold the mixing launches (or their absence): capture them again
  for (auto& kv : e->denoise_graphs) cudaGraphExecDestroy(kv.second);
  e->denoise_graphs.clear();
  e->denoise_launches.clear();
  e->kv_mix = false;
  if (!wk) return PI05_OK;
  const size_t cache = (size_t)L * e->max_batch * e->P * P5_HD * 2;
  if (!e->kmix && (!dalloc(e, (void**)&e->kmix, cache) || !dalloc(e, (void**)&e->vmix, cache))) return PI05_ERR_CUDA;
  if (!e->mix_w && (!dalloc(e, (void**)&e->mix_w, (size_t)2 * L * L * 4) ||
                    !dalloc(e, (void**)&e->mix_b, (size_t)2 * L * P5_HD * 4)))
    return PI05_ERR_CUDA;
  // the Dense weights of the mixing are bf16: round on the way in
  std::vector<float> w((size_t)2 * L * L), b((size_t)2 * L * P5_HD);
  for (int i = 0; i < L * L; ++i) {
    w[i] = p5_round_bf(wk[i]);
    w[L * L + i] = p5_round_bf(wv[i]);
  }
  for (int i = 0; i < L * P5_HD; ++i) {
    b[i] = p5_round_bf(bk[i]);
    b[(size_t)L * P5_HD + i] = p5_round_bf(bv[i]);
  }
  if (cudaMemcpy(e->mix_w, w.data(), w.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->mix_b, b.data(), b.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return PI05_ERR_CUDA;
  e->kv_mix = true;
  return PI05_OK;
}

int pi05_set_inpaint_known(pi05_engine* e, int sample, const float* known) {
  if (!e || sample < 0 || sample >= e->max_batch) return PI05_ERR_ARG;
  if (!e->inp_fixed) {
    set_err(e, "pi05_set_inpaint_known: inpainting is off (call pi05_set_inpaint first)");
    return PI05_ERR_STATE;
  }
  cudaSetDevice(e->device);
  const int K = e->inp_fixed * P5_ACT_D, on = known ? 1 : 0;
  if (known && cudaMemcpyAsync(e->inp_known + (size_t)sample * K, known, (size_t)K * 4, cudaMemcpyDefault,
                               e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  if (cudaMemcpyAsync(e->inp_on + sample, &on, sizeof(int), cudaMemcpyHostToDevice, e->stream) != cudaSuccess)
    return PI05_ERR_CUDA;
  return pi05_sync(e);
}

int pi05_act(pi05_engine* e, int slot, const pi05_frame* frames, const int32_t* tokens, const float* state,
             const float* noise, float* out) {
  return pi05_act_batch(e, 1, &slot, frames, tokens, state, noise, out);
}

int pi05_reset_slot(pi05_engine* e, int slot) {
  if (!e || slot < 0 || slot >= e->max_batch) return PI05_ERR_ARG;
  if ((int)e->act_chunk.size() == e->max_batch) {
    e->act_chunk[slot].clear();
    e->act_next[slot] = 0;
  }
  return PI05_OK;
}

}  // extern "C"

/*
 * pi05_oracle.h — CPU oracle for the pi0.5 engine path.  TEST INFRASTRUCTURE ONLY.
 *
 * This is an fp32 restatement of the pi0.5 network (SigLIP So400m/14 -> Gemma-2B prefix prefill ->
 * 10-step flow-matching denoise of the Gemma-300M action expert, plus the LoRA loss/gradient),
 * written from the model facts recorded in the reference (docs/archive/windows/π05_네이티브엔진.md:22-40,
 * :206-229) and the openpi code paths that record cites (models/pi0.py, models/gemma.py,
 * models/siglip.py, models/lora.py).  Activations are stored in bf16 at the points where the JAX
 * bf16 inference path rounds (the reference engine matched those points bit for bit,
 * π05_네이티브엔진.md:38-40); all arithmetic is fp32.  Setting P5O_FP32_ACTIVATIONS in `flags` keeps
 * every activation in fp32 instead (a pure-fp32 network on the same bf16 weights).
 *
 * Parity status: the reference engine's source and its golden dumps were deleted from the reference
 * repository, so this oracle is pinned only to the rounding conventions and shapes the record
 * states.  Only tests, the smoke check and the CPU-baseline leg of the benchmark may call it.
 */
#ifndef PI05_ORACLE_H
#define PI05_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t siglip_layers, gemma_layers, expert_layers, num_steps;
  int32_t n_cameras, n_text, horizon;
} p5o_config;

/* P5O_TEXT_PAD_MASK: a prompt's trailing ids 0 are padding, masked as openpi masks it: p5o_prefill's
 * queries attend to the first p5o_valid_prefix() keys only, and the denoise is then run on that many
 * cache rows (its action tokens' positions follow them). */
enum { P5O_FP32_ACTIVATIONS = 1, P5O_TEXT_PAD_MASK = 2 };
/* Two attention groups in the prefix (the PiBehavior variant's image + base-task block): flags carrying
 * P5O_PREFIX_GROUP(g) make prefix queries t < g attend to the keys j < g only; the others, and the action
 * tokens, attend to the whole prefix. */
#define P5O_PREFIX_GROUP(g) ((int)(g) << 16)
static inline int p5o_prefix_group(int flags) { return (flags >> 16) & 0x7fff; }

/* Named intermediate points (names follow the reference verifier: img.tokens, pre.lN.k, suf.sN.v, ...). */
typedef void (*p5o_probe_fn)(const char* name, const float* data, int64_t n, void* ctx);

int p5o_threads(void);

/* synthetic workload generators (streams shared with the engine) */
void p5o_gen_images(uint64_t seed, int sample, int n_cam, uint8_t* out);
void p5o_gen_tokens(uint64_t seed, int sample, int n, int32_t* out);
void p5o_gen_normal(uint64_t seed, int kind, int sub, int64_t n, double stdv, int round_bf16, float* out);
void p5o_gen_param(uint64_t seed, int kind, int sub, int64_t n, double stdv, float* out);
/* elements [first, first + n) of a parameter stream (rows of the token-embedding table) */
void p5o_gen_param_at(uint64_t seed, int kind, int sub, int64_t first, int64_t n, double stdv, float* out);

/* images: [n_cameras][224][224][3] uint8; out: [n_cameras*256][2048] */
int p5o_siglip(const p5o_config* c, uint64_t seed, const uint8_t* images, float* img_tokens, int flags,
               p5o_probe_fn probe, void* ctx);
/* prefix tokens attended to: P, or with P5O_TEXT_PAD_MASK the image tokens + the prompt before its padding */
int p5o_valid_prefix(const p5o_config* c, const int32_t* tokens, int flags);
/* full prefix: kcache/vcache [gemma_layers][P][256], P = 256*n_cameras + n_text */
int p5o_prefill(const p5o_config* c, uint64_t seed, const uint8_t* images, const int32_t* tokens,
                float* kcache, float* vcache, int flags, p5o_probe_fn probe, void* ctx);
/* prefix embeddings [P][2048]: SigLIP image tokens followed by the scaled text embeddings */
int p5o_prefix_embed(const p5o_config* c, uint64_t seed, const uint8_t* images, const int32_t* tokens, float* out,
                     int flags);
/* prefix given as embeddings [P][2048] (skips SigLIP and the text gather) */
int p5o_prefill_embedded(const p5o_config* c, uint64_t seed, const float* prefix_emb, int P,
                         float* kcache, float* vcache, int flags, p5o_probe_fn probe, void* ctx);
/* denoise: noise [horizon][32] -> actions [horizon][32] */
int p5o_denoise(const p5o_config* c, uint64_t seed, const float* kcache, const float* vcache, int P,
                const float* noise, float* actions, int flags, p5o_probe_fn probe, void* ctx);
/* denoise with soft inpainting: after each Euler step starting above t_min and landing at t, the first
 * fixed*32 values x_K <- t noise_K + (1 - t) known, and x_U += corr . (x_K,new - x_K,old);
 * known [fixed][32], corr [(horizon - fixed)*32][fixed*32] */
int p5o_denoise_inpaint(const p5o_config* c, uint64_t seed, const float* kcache, const float* vcache, int P,
                        const float* noise, float* actions, int flags, int fixed, float t_min, const float* known,
                        const float* corr);

#ifdef __cplusplus
}
#endif
#endif

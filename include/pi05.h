/*
 * pi05.h — C ABI of the B200-native pi0.5 engine (libpi05.so).
 *
 * Replaces the reference engine's batch API `include/pi05_batch.h` (deleted from the reference
 * repository; described in docs/archive/windows/π05_네이티브엔진.md:288-303 and :159) and its
 * training entry points `LoraTrainer::accumulate / finalize_grads / opt_step`
 * (π05_네이티브엔진.md:215).  Error convention follows the reference's other C ABIs
 * (src/scene_graph/runtime/include/sgrt.h:31-40): opaque handle, `char* err, size_t err_len` on
 * create, `int` status (0 = success, negative = failure) and a last-error accessor.
 *
 * Pointers: every input/output buffer may be a host pointer or a CUDA device pointer of the
 * engine's device (detected per call).  With host outputs the call returns after the result is in
 * host memory; with device outputs the work is only stream-ordered on the engine stream
 * (pi05_stream) and pi05_sync waits for it.  Calls on one engine are not re-entrant.
 *
 * Shapes (n = batch of independent observations, n <= max_batch):
 *   images   uint8 [n][n_cameras][224][224][3]  (RGB 224x224; pi05_act_batch takes camera frames of any size)
 *   tokens   int32 [n][n_text]                  (ids < 257152)
 *   noise    fp32  [n][horizon][32]             (flow-matching start x_1)
 *   actions  fp32  [n][horizon][32]             (x_0 after num_steps Euler steps)
 *   prefix KV cache bf16 (uint16 bits) [n][layers][P][256] each for K and V, P = 256*n_cameras + n_text
 */
#ifndef PI05_H
#define PI05_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PI05_API __attribute__((visibility("default")))
#else
#define PI05_API
#endif

#define PI05_OK 0
#define PI05_ERR_ARG (-1)     /* bad argument or shape */
#define PI05_ERR_CUDA (-2)    /* CUDA runtime error */
#define PI05_ERR_STATE (-3)   /* call out of order (e.g. denoise before prefill) */
#define PI05_ERR_DEVICE (-4)  /* a device-side wait gave up (lost arrival); the engine stays usable */

typedef struct pi05_engine pi05_engine;

/* Model hyper-parameters (the reference read these from `cfg` lines of its weight manifest,
 * π05_네이티브엔진.md:47).  Widths are fixed by the architecture; depths may be reduced for tests. */
typedef struct {
  int32_t siglip_layers;   /* 27 */
  int32_t gemma_layers;    /* 18 */
  int32_t expert_layers;   /* 18, must equal gemma_layers (expert layer l reads prefix layer l's KV) */
  int32_t num_steps;       /* 10 Euler steps, t = 1 -> 0 */
  int32_t n_cameras;       /* 3 */
  int32_t n_text;          /* 200 prompt tokens */
  int32_t horizon;         /* 50 actions per chunk */
  /* 1: every sample of a batch is computed exactly as a batch of one (at its own offsets, one
   * single-sample CUDA graph per batch position), so results are bit-identical for any batch size and
   * position, as the reference's batch path was (π05_네이티브엔진.md:299-302), at about the bs1 throughput.
   * 0 (default): batches run as one GEMM/attention problem each, for throughput; per-sample results
   * then differ from the batch-of-one results in the last bits (different tilings and sum orders). */
  int32_t batch_invariant;
  /* 1: a prompt shorter than n_text is padded with id 0 (openpi's padding, pi05_tokenize_prompt's output)
   * and masked as openpi masks it: no query attends to the padding, and the action tokens' RoPE positions
   * follow the last real token; each sample's length is read from its tokens on the device.  0 (default):
   * all n_text prompt positions are attended to (the benchmarks' full 200-token prompts).  Inference only
   * (pi05_lora_init refuses it), and it needs the tensor-core attention and the fused RoPE projections. */
  int32_t text_pad_mask;
  /* > 0: two attention groups in the prefix, as the PiBehavior variant's images + base task block
   * (π05_네이티브엔진.md:138, "softmax kernel with a group-boundary argument"): prefix queries t < prefix_group
   * attend to the prefix keys j < prefix_group only; the later prefix tokens and the action tokens attend
   * to the whole prefix.  0 (default): one group.  Inference only, on the tensor-core attention. */
  int32_t prefix_group;
} pi05_config;

PI05_API void pi05_default_config(pi05_config* c);

/* Replaces pi05_create_batch(weights, device, max_batch) (π05_네이티브엔진.md:290). */
PI05_API pi05_engine* pi05_create(const pi05_config* c, int device, int max_batch, char* err, size_t err_len);
PI05_API void pi05_destroy(pi05_engine* e);
PI05_API const char* pi05_last_error(const pi05_engine* e);

/* Weights.  pi05_init_random_weights fills every tensor from the seeded generator (linear weights
 * N(0, 0.02) in bf16; the synthetic workload of the benchmarks).  Weight files (.pi05w, the reference's
 * scheme, π05_네이티브엔진.md:46-49): a text manifest of "cfg <key> <value>" lines (the pi05_config fields)
 * and "t <name> <bf16|f32> <offset> <bytes> <dims...>" lines, then 256-byte aligned raw tensors, every
 * linear [out][in].  pi05_save_weights writes the engine's layout (bf16, fused q|k|v, gate/up rows
 * interleaved).  pi05_load_weights also takes the reference's layout, tensor by tensor (:48): separate
 * q/k/v and gate/up tensors (interleaved on load; q/k rows are paired per head for the fused RoPE when
 * the engine prepares them), the SigLIP MLP padded 4304 -> 4352 (padding dropped), the 588-column patch
 * embedding, one adaRMS Dense per norm, f32 tensors rounded to bf16 (the reference cast its f32
 * checkpoint the same way, :32); a file whose cfg differs from the engine's is refused.
 * pi05_read_weights_config: the file's configuration (defaults for keys it lacks), no GPU needed. */
PI05_API int pi05_init_random_weights(pi05_engine* e, uint64_t seed);
PI05_API int pi05_save_weights(pi05_engine* e, const char* path);
PI05_API int pi05_load_weights(pi05_engine* e, const char* path);
PI05_API int pi05_read_weights_config(const char* path, pi05_config* c);

/* Prefix: SigLIP over the camera images, text embedding, Gemma-2B prefill; fills the per-sample
 * bf16 KV cache.  (Reference: the per-board prefix CUDA graph, π05_네이티브엔진.md:298.) */
PI05_API int pi05_prefill(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens);
/* pi05_prefill with the text part of the prefix given as embeddings instead of token ids: text_emb bf16
 * (uint16 bits) [n][n_text][2048], the Gemma prefix's rows after the image tokens, already
 * scaled as the model wants them (the token path's rows are embedding * sqrt(2048) rounded to bf16).  For
 * callers whose prompt is not a sentence: the reference's PiBehavior model replaced it with learned task
 * embeddings and stage tokens (π05_네이티브엔진.md:136-137), which the caller forms.  Host or device
 * pointers; text_pad_mask must be 0 (it reads token ids). */
PI05_API int pi05_prefill_embeds(pi05_engine* e, int n, const uint8_t* images, const uint16_t* text_emb);
/* Install a prefix KV cache directly (the expert-only denoise workload). */
PI05_API int pi05_set_prefix_cache(pi05_engine* e, int n, const uint16_t* k, const uint16_t* v);
/* Read one layer of one sample's prefix cache (K and V, [P][256] bf16 bits each). */
PI05_API int pi05_get_prefix_cache(pi05_engine* e, int sample, int layer, uint16_t* k, uint16_t* v);
/* Denoise: num_steps Euler steps of the action expert attending to the prefix cache. */
PI05_API int pi05_denoise(pi05_engine* e, int n, const float* noise, float* actions);
/* prefill + denoise (replaces pi05_infer_batch, π05_네이티브엔진.md:292). */
PI05_API int pi05_infer(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* noise,
               float* actions);

/* Verify run (replaces the reference's layer-by-layer verifier tools/verify.cpp, π05_네이티브엔진.md:53-63,
 * whose point names it keeps): one observation (batch 1) through the same kernels as pi05_infer,
 * launched one by one instead of from the CUDA graph, with each named intermediate point copied to
 * the host as fp32 and passed to `fn` in network order:
 *   img.stem, img.l<N>.out, img.encoded, img.tokens        [256*n_cameras][1152 or 2048]
 *   txt.emb                                                [n_text][2048]
 *   pre.l<N>.norm1, .k, .v, .norm2, .out                   [P][2048] or [P][256] (the last layer: norm1, k, v)
 *   suf.s<S>.in, .l<N>.out, .final                         [horizon][1024]
 *   suf.s<S>.v, .x                                         [horizon][32] (velocity, flow state after step S)
 * `data` is valid during the callback only.  `actions` (optional) receives the chunk, the same values
 * pi05_infer returns for this observation.  Inputs may be host or device pointers. */
typedef void (*pi05_probe_fn)(const char* name, const float* data, int64_t n, void* ctx);
PI05_API int pi05_verify(pi05_engine* e, const uint8_t* images, const int32_t* tokens, const float* noise,
                         float* actions, pi05_probe_fn fn, void* ctx);
/* Teacher-forced verify run (the reference verifier's one-layer mode, π05_네이티브엔진.md:53-56): as
 * pi05_verify, but `fn` may overwrite `data`; the values (rounded to bf16 for bf16 points) replace the
 * engine's before the next kernel reads them, so planting a reference's layer outputs (img.l<N>.out,
 * img.tokens, pre.l<N>.out, suf.s<S>.l<N>.out, suf.s<S>.x) makes every layer start from the reference's
 * input and shows each layer's own error.  The adaRMSNorm of the denoise runs as a separate kernel in
 * this mode (its fused form reads statistics made before the planting point). */
typedef void (*pi05_plant_fn)(const char* name, float* data, int64_t n, void* ctx);
PI05_API int pi05_verify_planted(pi05_engine* e, const uint8_t* images, const int32_t* tokens, const float* noise,
                                 float* actions, pi05_plant_fn fn, void* ctx);

/* Stream and synchronisation. */
PI05_API void* pi05_stream(pi05_engine* e);  /* cudaStream_t of the engine */
PI05_API int pi05_sync(pi05_engine* e);      /* waits for queued work; reports device-side errors */

/* Prefix length P for the configuration. */
PI05_API int pi05_prefix_len(const pi05_engine* e);
/* Kernels one call enqueues, counted when its CUDA graph was captured (which: 0 prefill, 1 denoise);
 * -1 before the first call with batch n. */
PI05_API long pi05_graph_launches(pi05_engine* e, int which, int n);

/* Synthetic workload (host): the generator streams the tests and benchmarks use. */
PI05_API void pi05_synth_images(uint64_t seed, int sample, int n_cameras, uint8_t* out);
PI05_API void pi05_synth_tokens(uint64_t seed, int sample, int n_text, int32_t* out);
PI05_API void pi05_synth_noise(uint64_t seed, int sample, int horizon, float* out);
/* Expert-only workload: N(0,1) bf16 prefix cache for samples [0, n) generated on the device. */
PI05_API int pi05_synth_prefix_cache(pi05_engine* e, int n, uint64_t seed);

/* ---- LoRA fine-tuning (replaces LoraTrainer::accumulate / finalize_grads / opt_step, π05_네이티브엔진.md:215) ----
 * Rank-16, alpha-32 adapters on q/k/v/o/gate/up/down of the Gemma-2B prefix and of the action expert;
 * base weights frozen.  Loss: flow-matching MSE on the velocity (openpi pi0.py:189-214) with
 * x_t = t*noise + (1-t)*actions, u = noise - actions; the caller draws t (Beta(1.5,1)*0.999+0.001)
 * and the noise.  Optimizer: global-norm clip, AdamW.  Adapter parameters and gradients are one flat
 * fp32 buffer (per stack, per layer, per projection: A [16][in] then B [out][16]). */
typedef struct {
  int32_t rank;        /* 16 */
  float alpha;         /* 32 */
  float lr;            /* 1e-4 */
  float beta1, beta2;  /* 0.9, 0.95 */
  float eps;           /* 1e-8 */
  float weight_decay;  /* 1e-10 */
  float clip_norm;     /* 1.0 (global norm) */
  int32_t micro_batch; /* samples per forward/backward pass; activations of all layers are kept */
  /* learning-rate schedule (openpi training/optimizer.py CosineDecaySchedule, the reference's recipe,
   * π05_네이티브엔진.md:216: warmup 1000, lr 2.5e-5, decay_steps 30000, decay_lr 2.5e-6): update k (k = 0, 1,
   * ..) uses lr * ... rising linearly from lr / (warmup + 1) over warmup_steps, then a half cosine from lr
   * to decay_lr at decay_steps; warmup_steps = decay_steps = 0 keeps lr constant (the default) */
  int32_t warmup_steps;
  int32_t decay_steps;
  float decay_lr;
  /* EMA of the adapters after every update, ema = d * ema + (1 - d) * params (openpi scripts/train.py,
   * the reference's 0.99, π05_네이티브엔진.md:216); 0 = none (the default) */
  float ema_decay;
} pi05_lora_config;
PI05_API void pi05_lora_default_config(pi05_lora_config* c);
/* The learning rate of update `k` (0-based) under c's schedule; host only. */
PI05_API float pi05_lora_schedule_lr(const pi05_lora_config* c, int k);
/* The EMA adapters (fp32 flat buffer, the layout of pi05_lora_get_params); PI05_ERR_STATE without EMA. */
PI05_API int pi05_lora_get_ema(pi05_engine* e, float* out);
/* Adapters initialised N(0, 0.01) from `seed`; needs weights loaded and max_batch >= micro_batch. */
PI05_API int pi05_lora_init(pi05_engine* e, const pi05_lora_config* c, uint64_t seed);
PI05_API long pi05_lora_num_params(pi05_engine* e);
PI05_API int pi05_lora_zero_grads(pi05_engine* e);
/* forward + backward over n samples into the flat gradient buffer (LoraTrainer::accumulate), which holds
 * the mean gradient over every sample accumulated since the last pi05_lora_zero_grads (calls of 8 + 8
 * samples give what one call of 16 gives, up to fp32 rounding);
 * images u8 [n][cams][224][224][3], tokens i32 [n][n_text], actions/noise f32 [n][horizon][32], t f32 [n];
 * *loss (optional) = mean squared velocity error over the samples accumulated since the last zero. */
PI05_API int pi05_lora_accumulate(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens,
                                  const float* actions, const float* noise, const float* t, float* loss);
/* global-norm clip + AdamW on the accumulated gradients (finalize_grads + opt_step).  For data
 * parallelism allreduce-average pi05_lora_grad_buffer across ranks between accumulate and this call. */
PI05_API int pi05_lora_opt_step(pi05_engine* e);
/* zero_grads + accumulate + opt_step */
PI05_API int pi05_lora_step(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* actions,
                            const float* noise, const float* t, float* loss);
/* Data parallelism over NCCL (the LoRA step's exchange: the adapter gradients, and the loss, averaged over
 * the ranks before the identical clip + AdamW on every rank; the reference trained on one GPU,
 * π05_네이티브엔진.md:464).  Rank 0 writes the 128-byte ncclUniqueId with pi05_nccl_unique_id and shares it
 * with the other ranks by any host channel; each rank then attaches its engine (one GPU per rank) after
 * pi05_lora_init.  Once attached, pi05_lora_step averages each layer's gradients on a communication
 * stream as soon as its backward pass has finished that layer (no host synchronisation), and
 * pi05_lora_opt_step averages the whole buffer first when the gradients came from pi05_lora_accumulate
 * calls.  Every rank takes the same calls in the same order.  NCCL is loaded at run time (libnccl.so.2,
 * the process's own copy when a framework has loaded one); waits on the communicator are bounded by
 * PI05_NCCL_TIMEOUT_S seconds (default 120).  pi05_lora_world: ranks of the attached communicator (1). */
PI05_API int pi05_nccl_unique_id(void* id);
PI05_API int pi05_lora_attach_nccl(pi05_engine* e, const void* id, int rank, int world);
PI05_API int pi05_lora_world(pi05_engine* e);
PI05_API int pi05_lora_get_params(pi05_engine* e, float* out);
PI05_API int pi05_lora_set_params(pi05_engine* e, const float* in);
PI05_API int pi05_lora_get_grads(pi05_engine* e, float* out);
PI05_API void* pi05_lora_grad_buffer(pi05_engine* e); /* device pointer to the fp32 gradients */
/* zero the AdamW moments and the step count */
PI05_API int pi05_lora_reset_optimizer(pi05_engine* e);
/* checkpoint / resume of the train state: adapters, AdamW moments, step and (when enabled) the EMA (fp32
 * flat buffers; the reference saved params, EMA, Adam m/v and step, π05_네이티브엔진.md:281-282) */
PI05_API int pi05_lora_save_state(pi05_engine* e, const char* path);
PI05_API int pi05_lora_load_state(pi05_engine* e, const char* path);

/* Hot operators on caller-owned device buffers, run on the engine stream (unit tests and the operator
 * sweep).  pi05_op_linear: out[T][F'] = epilogue(x[T][K] . w[F][K]^T) with bf16 x, w, out and
 *   epi 0 store, 1 gelu, 2 residual (res[T][F]), 3 gated residual (res, gate[F]), 4 GeGLU
 *   (w rows interleaved gate/up, F' = F/2), 5 fp32 out.  bias[F] optional (NULL).
 *   No counterpart in the reference's ABI: its GEMM (src/gemm.cuh, π05_네이티브엔진.md:102-105) was internal.
 * pi05_op_attention: out[b][t][8*256] = softmax(q k^T) v with q [b][T][ldq] (8 heads x 256 at column 0,
 *   already scaled), keys/values [b][S][256] bf16; `splits` key splits (0: the engine chooses, as inside
 *   pi05_denoise).  Asynchronous; call pi05_sync. */
PI05_API int pi05_op_linear(pi05_engine* e, int T, int F, int K, const void* x, const void* w, const void* bias,
                            const void* res, const void* gate, int epi, void* out);
PI05_API int pi05_op_attention(pi05_engine* e, int batch, int T, int S, const void* q, int ldq, const void* k,
                               const void* v, void* out, int splits);
/* SigLIP attention of `images` 256-token images: qkv [images*256][3*1152] (q | k | v, 16 heads x 72
 * each), out [images*256][1152] = softmax(R(q / sqrt(72)) k^T) v per head and image.  The vision
 * tower's own attention step (reference: SigLIP block in the pi05 engine, π05_네이티브엔진.md); exposed as
 * an operator for tests and benchmarks.  Asynchronous; call pi05_sync. */
PI05_API int pi05_op_siglip_attention(pi05_engine* e, int images, const void* qkv, void* out);
/* Device time (microseconds per launch) of pi05_op_linear on internal random operands: `reps` launches
 * in one CUDA graph, rotating over enough weight copies (> 256 MB) that each launch reads HBM. */
PI05_API int pi05_op_bench_linear(pi05_engine* e, int T, int F, int K, int epi, int reps, float* us_per_launch);

/* Few-token linear layer that allocates nothing: out[T][F] = bf16(x[T][K] . w[F][K]^T + bias[F]), the
 * same kernel and tiling as the engine's weight-streaming path, for callers that cannot call
 * cudaMalloc (a process whose device memory is owned by another allocator, a real-time loop that
 * must not allocate after start-up).  Its split-K scratch is one file-scope device array of
 * 16 MiB that every GPU loading this library holds until exit.  Limits: 1 <= T <= 64,
 * 1 <= F <= 65536, 8 <= K <= 65536, K % 8 == 0; other sizes return PI05_ERR_ARG with a message in err.
 * x, w and out are 16-byte aligned device pointers, bias a device pointer or NULL.
 * The first call on a device sets that device up (looks up the array's address) and should come
 * before any stream capture.  All calls share the array: calls that overlap on the GPU race.
 * Asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream).  The kernel's waits are
 * bounded; one that gives up leaves that call's output incomplete and makes later calls skip their
 * work until pi05_linear_static_status reports it.  No counterpart in the reference's ABI. */
PI05_API int pi05_linear_static(int T, int F, int K, const void* x, const void* w, const void* bias, void* out,
                                void* stream, char* err, size_t err_len);
/* Waits for `stream`, then reports (PI05_ERR_DEVICE, message in err) and clears a bounded-wait
 * give-up recorded by pi05_linear_static calls on the current device; PI05_OK when there was none.
 * No counterpart in the reference's ABI. */
PI05_API int pi05_linear_static_status(void* stream, char* err, size_t err_len);

/* Reference batch-API names (π05_네이티브엔진.md:288-303).  pi05_create_batch configures the engine from the
 * weight file's cfg lines (NULL path: default configuration with pi05_init_random_weights(0)). */
PI05_API pi05_engine* pi05_create_batch(const char* weights_path, int device, int max_batch);
PI05_API int pi05_infer_batch(pi05_engine* e, int n, const uint8_t* images, const int32_t* tokens, const float* noise,
                     float* actions);
/* PiBehavior stage channel; plain pi0.5 has no stage head, so this only validates its arguments. */
PI05_API int pi05_set_stage(pi05_engine* e, int slot, int stage, int mode);
/* Receding-horizon stepping (reference pi05_act_batch / pi05_act, π05_네이티브엔진.md:292-297, :33, :303).
 * A camera frame as the evaluator passes it: RGB or RGBA (alpha ignored) at any resolution, rows `stride`
 * bytes apart, in host memory or device memory of the engine's device.  Frames that are not 224x224 are
 * resized with padding on the GPU (resize_with_pad: the pi05_resize_with_pad arithmetic, bit for bit). */
typedef struct {
  const void* data;
  int32_t height, width;
  int32_t channels; /* 3 = RGB, 4 = RGBA */
  int64_t stride;   /* bytes from one row to the next, >= width * channels */
} pi05_frame;
/* Output transform and re-plan period of pi05_act_batch (the wrapper's, π05_네이티브엔진.md:32-35, :293-295):
 * each new chunk is un-normalised a = a * (std + 1e-6) + mean (openpi Unnormalize, z-score; mean/std NULL:
 * none), the state is added to the dims that delta_mask marks (openpi AbsoluteActions; NULL: none), and
 * the first act_dim dims are kept.  A slot re-plans when it has no chunk or has executed `replan` rows.
 * Noise, when the caller passes none, comes from the slot's own generator stream: re-plan p of slot s
 * draws elements [p, p+1) * horizon*32 of the stream (noise_seed, noise, s), so its first re-plan uses
 * pi05_synth_noise(noise_seed, s).  Setting the configuration forgets every slot's chunk.
 * Defaults: act_dim 32, replan 16, no transforms, noise_seed 0. */
typedef struct {
  int32_t act_dim;
  int32_t replan;
  const float* mean;          /* [act_dim] or NULL */
  const float* std;           /* [act_dim] or NULL */
  const uint8_t* delta_mask;  /* [act_dim] or NULL */
  uint64_t noise_seed;
} pi05_act_config;
PI05_API int pi05_set_act_config(pi05_engine* e, const pi05_act_config* c);
/* One environment step of the n slots slots[i] (each at most once per call): writes the slot's next
 * action row to out[i][act_dim] (f32, host or device), after one batched inference for the listed slots
 * that re-plan.  frames [n][n_cameras] (frames[i * n_cameras + c]); tokens int32 [n][n_text]; state f32
 * [n][act_dim] (read for the delta dims; may be NULL without a delta mask); noise f32 [n][horizon][32]
 * or NULL (the slots' generator streams).  Host or device pointers.  With batch_invariant = 1 the result
 * is bit-identical to stepping each slot alone with pi05_act. */
PI05_API int pi05_act_batch(pi05_engine* e, int n, const int* slots, const pi05_frame* frames, const int32_t* tokens,
                            const float* state, const float* noise, float* out);
/* Correlated noise for the re-plans whose noise the engine draws (pi05_act_batch with noise NULL): each
 * slot's standard-normal draw eps over the flattened chunk (index t*32 + j) becomes L . eps, L the
 * lower-triangular [dim][dim] factor of the covariance (dim = horizon * 32; the reference's PiBehavior
 * model drew N(0, 0.5 I + 0.5 Sigma) with a Cholesky factor computed in f64 at export, π05_네이티브엔진.md:141).
 * Accumulated in fp64 on the device.  L = NULL returns to uncorrelated noise. */
PI05_API int pi05_set_noise_cholesky(pi05_engine* e, const float* L, int dim);
/* Soft inpainting of the denoise (the reference's PiBehavior model, π05_네이티브엔진.md:142: the first four
 * actions of a chunk held to the ones already committed, only at flow times above 0.3, the rest corrected
 * through Sigma_UO Sigma_OO^-1, an 832 x 128 matrix computed at export).  With K = fixed * 32 and
 * U = horizon * 32 - K, after every Euler step that starts at a time t_s > t_min and lands at t, each batch
 * position whose known rows are on gets
 *   x[0:K] <- t eps[0:K] + (1 - t) known,   x[K:] += corr . (x[0:K],new - x[0:K],old)
 * eps the position's step-0 noise, corr f32 [U][K] row-major (host or device).  fixed = 0 switches
 * inpainting off; 1 <= fixed < horizon (and fixed <= 384).  Every position starts switched off.  A batch
 * position is the sample's index in a pi05_denoise / pi05_infer / pi05_infer_batch call. */
PI05_API int pi05_set_inpaint(pi05_engine* e, int fixed, float t_min, const float* corr);
/* KV layer mixing of the denoise (the reference's PiBehavior model, π05_네이티브엔진.md:140: "each action
 * expert layer sees a linear combination of the VLM's 18 layers' KV", computed as a bf16 einsum plus a bf16
 * bias): with L = gemma_layers, expert layer l attends to
 *   K~_l = bf16(bf16(sum_j wk[l][j] K_j) + bk[l]),   V~_l likewise with wv, bv
 * over the prefix cache's layers j (the action tokens' own K/V are not mixed).  wk, wv f32 [L][L] and bk, bv
 * f32 [L][256], host memory, rounded to bf16 on the way in; wk = NULL switches mixing off.  The mixed caches
 * are formed at the start of every pi05_denoise / pi05_infer call (one extra copy of the prefix cache is
 * allocated on first use); L <= 18; inference only (pi05_lora_init refuses it). */
PI05_API int pi05_set_kv_mix(pi05_engine* e, const float* wk, const float* bk, const float* wv, const float* bv);
/* The known rows of batch position `sample`: known f32 [fixed][32] in the model's (normalised) action
 * space, host or device; NULL switches the position back to free denoising. */
PI05_API int pi05_set_inpaint_known(pi05_engine* e, int sample, const float* known);
/* pi05_act_batch for one slot (the reference's single-slot pi05_act). */
PI05_API int pi05_act(pi05_engine* e, int slot, const pi05_frame* frames, const int32_t* tokens, const float* state,
                      const float* noise, float* out);
/* Forget a slot's chunk (reference reset(eng, slot)): its next pi05_act_batch step re-plans. */
PI05_API int pi05_reset_slot(pi05_engine* e, int slot);
/* Camera-frame preprocessing on the host (reference resize_with_pad, π05_네이티브엔진.md:296-297, after
 * openpi image_tools.resize_with_pad with Pillow's bilinear filter): the h x w frame (`channels` 3 = RGB
 * or 4 = RGBA, alpha dropped; rows `stride` bytes apart) is resized keeping its aspect ratio and pasted,
 * centred, into a zero out_h x out_w RGB frame (dst, out_h*out_w*3 bytes); a frame of the output size
 * is copied.  Host memory; needs no engine or GPU. */
PI05_API int pi05_resize_with_pad(const uint8_t* src, int h, int w, int channels, long stride, uint8_t* dst, int out_h,
                                  int out_w);
/* State / action transforms of the reference wrapper (π05_네이티브엔진.md:32-35, :83-84, after openpi's
 * Normalize, Unnormalize, AbsoluteActions and the pi0.5 state discretisation), float32, host memory:
 *   pi05_normalize: x[n][dim] in place; mode 0 z-score with (a, b) = (mean, std), mode 1 quantile with
 *     (a, b) = (q01, q99) mapping to [-1, 1]; inverse != 0 un-normalises;
 *   pi05_discretize_state: out[n][dim] = bin of x among `bins` equal bins of [-1, 1) (-1 below -1);
 *   pi05_absolute_actions: actions[horizon][dim] += state where mask != 0 (delta actions). */
PI05_API int pi05_normalize(float* x, int n, int dim, const float* a, const float* b, int mode, int inverse);
PI05_API int pi05_discretize_state(const float* x, int n, int dim, int bins, int32_t* out);
PI05_API int pi05_absolute_actions(float* actions, int horizon, int dim, const float* state, const uint8_t* mask);
/* PiBehavior wrapper helpers (π05_네이티브엔진.md:143, checked at :146), host memory, no engine needed:
 *   pi05_interp_actions_cubic: out[n_out][dim] = the not-a-knot cubic spline through in[n_in][dim] at the
 *     knots 0..n_in-1, sampled at k (n_in - 1) / (n_out - 1) (scipy interp1d kind="cubic"; n_in >= 4);
 *   pi05_stage_vote: the stage predicted at least twice among the last three of recent[n] (oldest first),
 *     else `current`; capped below max_stage when max_stage > 0.  Returns the stage (>= 0) or an error. */
PI05_API int pi05_interp_actions_cubic(const float* in, int n_in, int dim, float* out, int n_out);
PI05_API int pi05_stage_vote(const int32_t* recent, int n, int current, int max_stage);

/* Prompt tokenizer (the reference's C++ SentencePiece tokenizer, π05_네이티브엔진.md:83): a SentencePiece BPE
 * model read from its .model file (identity normalization, byte fallback, user-defined symbols; Gemma's
 * tokenizer is such a model; the file itself is not part of this build).  Host only, no GPU.
 *   pi05_tokenizer_encode: ids of `text` (BOS first when add_bos); returns the number of ids (only the
 *     first max_ids are written) or a negative error.
 *   pi05_tokenize_prompt: the pi0.5 prompt of openpi's PaligemmaTokenizer: the task stripped, '_' and
 *     newlines as spaces, "Task: <task>, State: <256-bin state bins>;\nAction: " with BOS, padded with 0 (mask
 *     0) or cut to max_len (n_text); state_dim = 0 gives the pi0 layout (task, BOS, then "\n").  Returns the
 *     number of real tokens. */
typedef struct pi05_tokenizer pi05_tokenizer;
PI05_API pi05_tokenizer* pi05_tokenizer_load(const char* model_path, char* err, size_t err_len);
PI05_API void pi05_tokenizer_free(pi05_tokenizer* t);
PI05_API int pi05_tokenizer_vocab_size(const pi05_tokenizer* t);
PI05_API int pi05_tokenizer_encode(const pi05_tokenizer* t, const char* text, int add_bos, int32_t* ids, int max_ids);
PI05_API int pi05_tokenize_prompt(const pi05_tokenizer* t, const char* task, const float* state, int state_dim,
                                  int max_len, int32_t* ids, uint8_t* mask);

#ifdef __cplusplus
}
#endif
#endif /* PI05_H */

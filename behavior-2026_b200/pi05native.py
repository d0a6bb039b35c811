"""Python binding of libpi05.so (include/pi05.h).

Mirrors the reference engine's CPython module `_pi05native` and its `Pi05NativePolicy` wrapper
(glue/pi05native_module.c, glue/pi05_policy.py in the deleted engine; described in
docs/archive/windows/π05_네이티브엔진.md:109-117): buffers are passed by pointer, numpy arrays as host
pointers, CUDA tensors (anything with ``__cuda_array_interface__`` or a torch CUDA tensor) as device
pointers without a copy.  ctypes releases the GIL during each call.

There is no fallback: if libpi05.so is missing or fails to load, importing this module raises.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpi05.so")

OK, ERR_ARG, ERR_CUDA, ERR_STATE, ERR_DEVICE = 0, -1, -2, -3, -4

EXPORTS = [
    "pi05_default_config", "pi05_create", "pi05_destroy", "pi05_last_error", "pi05_init_random_weights",
    "pi05_save_weights", "pi05_load_weights", "pi05_prefill", "pi05_set_prefix_cache", "pi05_get_prefix_cache",
    "pi05_denoise", "pi05_infer", "pi05_stream", "pi05_sync", "pi05_prefix_len", "pi05_graph_launches",
    "pi05_synth_images", "pi05_synth_tokens", "pi05_synth_noise", "pi05_synth_prefix_cache", "pi05_create_batch",
    "pi05_infer_batch", "pi05_set_stage", "pi05_act_batch", "pi05_reset_slot", "pi05_resize_with_pad", "pi05_normalize", "pi05_discretize_state", "pi05_absolute_actions", "pi05_interp_actions_cubic", "pi05_stage_vote", "pi05_op_linear", "pi05_op_attention", "pi05_op_siglip_attention", "pi05_linear_static",
    "pi05_linear_static_status", "pi05_verify", "pi05_set_act_config", "pi05_act",
    "pi05_nccl_unique_id", "pi05_lora_attach_nccl", "pi05_lora_world",
    "pi05_read_weights_config", "pi05_lora_schedule_lr", "pi05_lora_get_ema", "pi05_tokenizer_load",
    "pi05_tokenizer_free", "pi05_tokenizer_vocab_size", "pi05_tokenizer_encode", "pi05_tokenize_prompt",
    "pi05_set_noise_cholesky", "pi05_set_inpaint", "pi05_set_inpaint_known", "pi05_set_kv_mix", "pi05_prefill_embeds", "pi05_verify_planted",
]


class Pi05Error(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"pi05 error {code}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("siglip_layers", "gemma_layers", "expert_layers", "num_steps", "n_cameras", "n_text", "horizon",
                 "batch_invariant", "text_pad_mask", "prefix_group")]

    @classmethod
    def make(cls, siglip_layers=27, gemma_layers=18, num_steps=10, n_cameras=3, n_text=200, horizon=50,
             batch_invariant=0, text_pad_mask=0, prefix_group=0):
        return cls(siglip_layers, gemma_layers, gemma_layers, num_steps, n_cameras, n_text, horizon, batch_invariant,
                   text_pad_mask, prefix_group)

    @property
    def prefix_len(self):
        return 256 * self.n_cameras + self.n_text

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class Frame(ctypes.Structure):
    """pi05_frame: one camera frame (RGB or RGBA, any size and row stride, host or device memory)"""
    _fields_ = [("data", ctypes.c_void_p), ("height", ctypes.c_int32), ("width", ctypes.c_int32),
                ("channels", ctypes.c_int32), ("stride", ctypes.c_int64)]


class ActConfig(ctypes.Structure):
    _fields_ = [("act_dim", ctypes.c_int32), ("replan", ctypes.c_int32), ("mean", ctypes.c_void_p),
                ("std", ctypes.c_void_p), ("delta_mask", ctypes.c_void_p), ("noise_seed", ctypes.c_uint64)]


class LoraConfig(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("alpha", ctypes.c_float), ("lr", ctypes.c_float), ("beta1", ctypes.c_float),
                ("beta2", ctypes.c_float), ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float),
                ("clip_norm", ctypes.c_float), ("micro_batch", ctypes.c_int32), ("warmup_steps", ctypes.c_int32),
                ("decay_steps", ctypes.c_int32), ("decay_lr", ctypes.c_float), ("ema_decay", ctypes.c_float)]

    @classmethod
    def reference_recipe(cls, micro_batch=8):
        """the reference's fine-tuning recipe (π05_네이티브엔진.md:216): warmup 1000 -> cosine 2.5e-5 -> 2.5e-6 at
        30000 steps, EMA 0.99"""
        c = cls()
        lib.pi05_lora_default_config(ctypes.byref(c))
        c.micro_batch, c.lr, c.warmup_steps, c.decay_steps, c.decay_lr, c.ema_decay = micro_batch, 2.5e-5, 1000, \
            30000, 2.5e-6, 0.99
        return c


def lora_schedule_lr(config, k):
    """pi05_lora_schedule_lr: the learning rate of update k under `config` (a LoraConfig)"""
    return lib.pi05_lora_schedule_lr(ctypes.byref(config), k)


PROBE = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64, ctypes.c_void_p)
PLANT = PROBE  # same C signature; the data of a teacher-forced run may be written


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with behavior-2026_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    P, vp, i32, u64 = ctypes.POINTER, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    cfg = P(Config)
    L.pi05_default_config.argtypes = [cfg]
    L.pi05_default_config.restype = None
    L.pi05_create.argtypes = [cfg, i32, i32, ctypes.c_char_p, ctypes.c_size_t]
    L.pi05_create.restype = vp
    L.pi05_destroy.argtypes = [vp]
    L.pi05_destroy.restype = None
    L.pi05_last_error.argtypes = [vp]
    L.pi05_last_error.restype = ctypes.c_char_p
    L.pi05_init_random_weights.argtypes = [vp, u64]
    L.pi05_save_weights.argtypes = [vp, ctypes.c_char_p]
    L.pi05_load_weights.argtypes = [vp, ctypes.c_char_p]
    L.pi05_prefill.argtypes = [vp, i32, vp, vp]
    L.pi05_set_prefix_cache.argtypes = [vp, i32, vp, vp]
    L.pi05_get_prefix_cache.argtypes = [vp, i32, i32, vp, vp]
    L.pi05_denoise.argtypes = [vp, i32, vp, vp]
    L.pi05_infer.argtypes = [vp, i32, vp, vp, vp, vp]
    L.pi05_stream.argtypes = [vp]
    L.pi05_stream.restype = vp
    L.pi05_sync.argtypes = [vp]
    L.pi05_prefix_len.argtypes = [vp]
    L.pi05_graph_launches.argtypes = [vp, i32, i32]
    L.pi05_graph_launches.restype = ctypes.c_long
    L.pi05_synth_images.argtypes = [u64, i32, i32, vp]
    L.pi05_synth_tokens.argtypes = [u64, i32, i32, vp]
    L.pi05_synth_noise.argtypes = [u64, i32, i32, vp]
    for f in (L.pi05_synth_images, L.pi05_synth_tokens, L.pi05_synth_noise):
        f.restype = None
    L.pi05_synth_prefix_cache.argtypes = [vp, i32, u64]
    L.pi05_create_batch.argtypes = [ctypes.c_char_p, i32, i32]
    L.pi05_create_batch.restype = vp
    L.pi05_infer_batch.argtypes = [vp, i32, vp, vp, vp, vp]
    L.pi05_set_stage.argtypes = [vp, i32, i32, i32]
    L.pi05_act_batch.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    L.pi05_reset_slot.argtypes = [vp, i32]
    L.pi05_resize_with_pad.argtypes = [vp, i32, i32, i32, ctypes.c_long, vp, i32, i32]
    L.pi05_normalize.argtypes = [vp, i32, i32, vp, vp, i32, i32]
    L.pi05_discretize_state.argtypes = [vp, i32, i32, i32, vp]
    L.pi05_absolute_actions.argtypes = [vp, i32, i32, vp, vp]
    L.pi05_interp_actions_cubic.argtypes = [vp, i32, i32, vp, i32]
    L.pi05_stage_vote.argtypes = [vp, i32, i32, i32]
    L.pi05_op_linear.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, vp, i32, vp]
    L.pi05_op_attention.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp, vp, i32]
    L.pi05_op_siglip_attention.argtypes = [vp, i32, vp, vp]
    L.pi05_linear_static.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_char_p, ctypes.c_size_t]
    L.pi05_linear_static_status.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
    L.pi05_lora_default_config.argtypes = [P(LoraConfig)]
    L.pi05_lora_default_config.restype = None
    L.pi05_lora_schedule_lr.argtypes = [P(LoraConfig), i32]
    L.pi05_lora_schedule_lr.restype = ctypes.c_float
    L.pi05_lora_get_ema.argtypes = [vp, vp]
    L.pi05_lora_init.argtypes = [vp, P(LoraConfig), u64]
    L.pi05_lora_num_params.argtypes = [vp]
    L.pi05_lora_num_params.restype = ctypes.c_long
    L.pi05_lora_zero_grads.argtypes = [vp]
    L.pi05_lora_accumulate.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    L.pi05_lora_opt_step.argtypes = [vp]
    L.pi05_lora_step.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    L.pi05_lora_get_params.argtypes = [vp, vp]
    L.pi05_lora_set_params.argtypes = [vp, vp]
    L.pi05_lora_get_grads.argtypes = [vp, vp]
    L.pi05_lora_grad_buffer.argtypes = [vp]
    L.pi05_lora_grad_buffer.restype = vp
    L.pi05_op_bench_linear.argtypes = [vp, i32, i32, i32, i32, i32, P(ctypes.c_float)]
    L.pi05_lora_reset_optimizer.argtypes = [vp]
    L.pi05_verify.argtypes = [vp, vp, vp, vp, vp, PROBE, vp]
    L.pi05_verify_planted.argtypes = [vp, vp, vp, vp, vp, PLANT, vp]
    L.pi05_set_act_config.argtypes = [vp, P(ActConfig)]
    L.pi05_nccl_unique_id.argtypes = [vp]
    L.pi05_read_weights_config.argtypes = [ctypes.c_char_p, cfg]
    L.pi05_tokenizer_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
    L.pi05_tokenizer_load.restype = vp
    L.pi05_tokenizer_free.argtypes = [vp]
    L.pi05_tokenizer_free.restype = None
    L.pi05_tokenizer_vocab_size.argtypes = [vp]
    L.pi05_tokenizer_encode.argtypes = [vp, ctypes.c_char_p, i32, vp, i32]
    L.pi05_tokenize_prompt.argtypes = [vp, ctypes.c_char_p, vp, i32, i32, vp, vp]
    L.pi05_lora_attach_nccl.argtypes = [vp, vp, i32, i32]
    L.pi05_lora_world.argtypes = [vp]
    L.pi05_act.argtypes = [vp, i32, vp, vp, vp, vp, vp]
    L.pi05_set_noise_cholesky.argtypes = [vp, vp, i32]
    L.pi05_set_inpaint.argtypes = [vp, i32, ctypes.c_float, vp]
    L.pi05_set_inpaint_known.argtypes = [vp, i32, vp]
    L.pi05_set_kv_mix.argtypes = [vp, vp, vp, vp, vp]
    L.pi05_prefill_embeds.argtypes = [vp, i32, vp, vp]
    L.pi05_lora_save_state.argtypes = [vp, ctypes.c_char_p]
    L.pi05_lora_load_state.argtypes = [vp, ctypes.c_char_p]
    return L


lib = _load()


def _ptr(a, dtype=None, writable=False):
    """(pointer, keepalive) for a numpy array, a torch tensor or a __cuda_array_interface__ object."""
    if hasattr(a, "data_ptr") and hasattr(a, "is_contiguous"):  # torch tensor
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return ctypes.c_void_p(a.data_ptr()), a
    if hasattr(a, "__cuda_array_interface__"):
        return ctypes.c_void_p(a.__cuda_array_interface__["data"][0]), a
    arr = np.asarray(a)
    if dtype is not None and arr.dtype != dtype:
        if writable:
            raise ValueError(f"output array must be {dtype}")
        arr = arr.astype(dtype)
    if not arr.flags["C_CONTIGUOUS"]:
        if writable:
            raise ValueError("output array must be C-contiguous")
        arr = np.ascontiguousarray(arr)
    return ctypes.c_void_p(arr.ctypes.data), arr


class Engine:
    """One engine per device (reference: one engine, its own stream, graph captured at load)."""

    def __init__(self, config=None, device=0, max_batch=1):
        self.config = config if config is not None else Config.make()
        self.max_batch = max_batch
        err = ctypes.create_string_buffer(1024)
        h = lib.pi05_create(ctypes.byref(self.config), device, max_batch, err, len(err))
        if not h:
            raise Pi05Error(ERR_CUDA, err.value.decode())
        self._h = ctypes.c_void_p(h)

    # -- lifecycle
    def close(self):
        if getattr(self, "_h", None):
            lib.pi05_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def _check(self, rc):
        if rc != OK:
            raise Pi05Error(rc, lib.pi05_last_error(self._h).decode())

    @property
    def prefix_len(self):
        return lib.pi05_prefix_len(self._h)

    @property
    def stream(self):
        return lib.pi05_stream(self._h)

    def sync(self):
        self._check(lib.pi05_sync(self._h))

    def graph_launches(self, which, n):
        return lib.pi05_graph_launches(self._h, {"prefill": 0, "denoise": 1}.get(which, which), n)

    # -- weights
    def init_random_weights(self, seed=0):
        self._check(lib.pi05_init_random_weights(self._h, seed))

    def save_weights(self, path):
        self._check(lib.pi05_save_weights(self._h, path.encode()))

    def load_weights(self, path):
        self._check(lib.pi05_load_weights(self._h, path.encode()))

    # -- path
    def prefill(self, images, tokens):
        n = images.shape[0]
        pi, ki = _ptr(images, np.uint8)
        pt, kt = _ptr(tokens, np.int32)
        self._check(lib.pi05_prefill(self._h, n, pi, pt))

    def prefill_embeds(self, images, text_emb):
        """pi05_prefill_embeds: the prefix from the images and the text part's embeddings ([n][n_text][2048],
        bf16 bits as uint16, or float32 rounded to bf16 here)"""
        n = images.shape[0]
        emb = np.asarray(text_emb)
        if emb.dtype != np.uint16:
            emb = f32_to_bf16_bits(emb)
        if emb.shape != (n, self.config.n_text, 2048):
            raise ValueError(f"text_emb must be [{n}][{self.config.n_text}][2048], got {emb.shape}")
        emb = np.ascontiguousarray(emb)
        pi, ki = _ptr(images, np.uint8)
        self._check(lib.pi05_prefill_embeds(self._h, n, pi, emb.ctypes.data))

    def set_prefix_cache(self, k_bits, v_bits):
        """k_bits/v_bits: uint16 (bf16 bit patterns) [n][layers][P][256]."""
        n = k_bits.shape[0]
        pk, kk = _ptr(k_bits, np.uint16)
        pv, kv = _ptr(v_bits, np.uint16)
        self._check(lib.pi05_set_prefix_cache(self._h, n, pk, pv))

    def synth_prefix_cache(self, n, seed=0):
        self._check(lib.pi05_synth_prefix_cache(self._h, n, seed))

    def get_prefix_cache(self, sample, layer):
        P = self.prefix_len
        k = np.empty((P, 256), np.uint16)
        v = np.empty((P, 256), np.uint16)
        self._check(lib.pi05_get_prefix_cache(self._h, sample, layer, k.ctypes.data, v.ctypes.data))
        return bf16_bits_to_f32(k), bf16_bits_to_f32(v)

    def denoise(self, noise, out=None):
        n = noise.shape[0]
        if out is None:
            out = np.empty((n, self.config.horizon, 32), np.float32)
        pn, kn = _ptr(noise, np.float32)
        po, ko = _ptr(out, np.float32, writable=True)
        self._check(lib.pi05_denoise(self._h, n, pn, po))
        return out

    def infer_batch(self, images, tokens, noise, out=None):
        """pi05_infer_batch (the reference's name for infer)"""
        n = images.shape[0]
        if out is None:
            out = np.empty((n, self.config.horizon, 32), np.float32)
        pi, ki = _ptr(images, np.uint8)
        pt, kt = _ptr(tokens, np.int32)
        pn_, kn = _ptr(noise, np.float32)
        po, ko = _ptr(out, np.float32, writable=True)
        self._check(lib.pi05_infer_batch(self._h, n, pi, pt, pn_, po))
        return out

    def infer(self, images, tokens, noise, out=None):
        n = images.shape[0]
        if out is None:
            out = np.empty((n, self.config.horizon, 32), np.float32)
        pi, ki = _ptr(images, np.uint8)
        pt, kt = _ptr(tokens, np.int32)
        pn, kn = _ptr(noise, np.float32)
        po, ko = _ptr(out, np.float32, writable=True)
        self._check(lib.pi05_infer(self._h, n, pi, pt, pn, po))
        return out

    def verify(self, images, tokens, noise, keep=None):
        """Verify run of one observation (pi05_verify): returns (actions [horizon][32], {point name: fp32
        array}) with the points whose names start with one of `keep` (all when None): img.*, txt.emb,
        pre.l<N>.{norm1,k,v,norm2,out}, suf.s<S>.{in,l<N>.out,final,v,x}."""
        points = {}

        def on(name, data, n, _ctx):
            name = name.decode()
            if keep is None or any(name.startswith(k) for k in keep):
                points[name] = np.ctypeslib.as_array(data, shape=(n,)).copy()

        cb = PROBE(on)
        out = np.empty((self.config.horizon, 32), np.float32)
        pi, ki = _ptr(images, np.uint8)
        pt, kt = _ptr(tokens, np.int32)
        pn, kn = _ptr(noise, np.float32)
        self._check(lib.pi05_verify(self._h, pi, pt, pn, out.ctypes.data, cb, None))
        return out, points

    def verify_planted(self, images, tokens, noise, plant, keep=None):
        """Teacher-forced verify run (pi05_verify_planted): at every point named in `plant` ({name: array}) the
        engine's own value is recorded and then replaced by the planted one, so the next layer starts from it.
        Returns (actions, {name: the engine's value before planting, for planted points; the emitted value
        for other points whose names start with one of `keep`})."""
        seen = {}

        def on(name, data, n, _ctx):
            name = name.decode()
            arr = np.ctypeslib.as_array(data, shape=(n,))
            if name in plant:
                seen[name] = arr.copy()
                src = np.ascontiguousarray(plant[name], np.float32).reshape(-1)
                assert src.size == n, (name, src.size, n)
                arr[:] = src
            elif keep is not None and any(name.startswith(k) for k in keep):
                seen[name] = arr.copy()

        cb = PLANT(on)
        out = np.empty((self.config.horizon, 32), np.float32)
        pi, ki = _ptr(images, np.uint8)
        pt, kt = _ptr(tokens, np.int32)
        pn_, kn = _ptr(noise, np.float32)
        self._check(lib.pi05_verify_planted(self._h, pi, pt, pn_, out.ctypes.data, cb, None))
        return out, seen

    # -- hot operators on device tensors (asynchronous on the engine stream)
    EPI = {"store": 0, "gelu": 1, "resid": 2, "gated": 3, "geglu": 4, "f32": 5}

    def op_linear(self, x, w, out, epi="store", bias=None, res=None, gate=None):
        T, K = x.shape
        F = w.shape[0]
        p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
        self._check(lib.pi05_op_linear(self._h, T, F, K, p(x), p(w), p(bias), p(res), p(gate), self.EPI[epi], p(out)))

    def op_bench_linear(self, T, F, K, epi="store", reps=50):
        """device microseconds per launch of one linear layer (graph-timed, weights streamed from HBM)"""
        us = ctypes.c_float(0)
        self._check(lib.pi05_op_bench_linear(self._h, T, F, K, self.EPI[epi], reps, ctypes.byref(us)))
        return us.value

    def op_attention(self, q, k, v, out, splits=1):
        """q [b][T][ldq] (heads at column 0), k/v [b][S][256], out [b][T][2048]; all CUDA bf16 tensors.
        splits = 0 lets the engine choose the key splits (as inside pi05_denoise)."""
        b, T, ldq = q.shape
        S = k.shape[1]
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        self._check(lib.pi05_op_attention(self._h, b, T, S, p(q), ldq, p(k), p(v), p(out), splits))

    def op_siglip_attention(self, qkv, out):
        """qkv [images*256][3456] (q | k | v, 16 heads x 72), out [images*256][1152]; CUDA bf16 tensors."""
        images = qkv.shape[0] // 256
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        self._check(lib.pi05_op_siglip_attention(self._h, images, p(qkv), p(out)))

    # -- LoRA fine-tuning (reference: LoraTrainer::accumulate / finalize_grads / opt_step)
    def lora_init(self, seed=0, micro_batch=8, **kw):
        c = LoraConfig()
        lib.pi05_lora_default_config(ctypes.byref(c))
        c.micro_batch = micro_batch
        for k, v in kw.items():
            setattr(c, k, v)
        self._check(lib.pi05_lora_init(self._h, ctypes.byref(c), seed))
        self.lora_config = c

    @property
    def lora_num_params(self):
        return lib.pi05_lora_num_params(self._h)

    def lora_zero_grads(self):
        self._check(lib.pi05_lora_zero_grads(self._h))

    def _lora_args(self, images, tokens, actions, noise, t):
        keep = [_ptr(images, np.uint8), _ptr(tokens, np.int32), _ptr(actions, np.float32), _ptr(noise, np.float32),
                _ptr(t, np.float32)]
        return [k[0] for k in keep], keep

    def lora_accumulate(self, images, tokens, actions, noise, t):
        """forward + backward; adds to the gradient buffer; returns the running mean loss"""
        ptrs, keep = self._lora_args(images, tokens, actions, noise, t)
        loss = ctypes.c_float(0)
        self._check(lib.pi05_lora_accumulate(self._h, images.shape[0], *ptrs, ctypes.byref(loss)))
        return loss.value

    def lora_opt_step(self):
        self._check(lib.pi05_lora_opt_step(self._h))

    def lora_step(self, images, tokens, actions, noise, t, want_loss=True):
        ptrs, keep = self._lora_args(images, tokens, actions, noise, t)
        loss = ctypes.c_float(0)
        self._check(lib.pi05_lora_step(self._h, images.shape[0], *ptrs, ctypes.byref(loss) if want_loss else None))
        return loss.value

    def lora_get_params(self):
        out = np.empty(self.lora_num_params, np.float32)
        self._check(lib.pi05_lora_get_params(self._h, out.ctypes.data))
        return out

    def lora_set_params(self, p):
        p = np.ascontiguousarray(p, np.float32)
        self._check(lib.pi05_lora_set_params(self._h, p.ctypes.data))

    def lora_get_ema(self):
        out = np.empty(self.lora_num_params, np.float32)
        self._check(lib.pi05_lora_get_ema(self._h, out.ctypes.data))
        return out

    def lora_get_grads(self):
        out = np.empty(self.lora_num_params, np.float32)
        self._check(lib.pi05_lora_get_grads(self._h, out.ctypes.data))
        return out

    def lora_grad_ptr(self):
        return lib.pi05_lora_grad_buffer(self._h)

    def lora_attach_nccl(self, unique_id, rank, world):
        """pi05_lora_attach_nccl: join the `world`-rank communicator of the 128-byte NCCL id"""
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        self._check(lib.pi05_lora_attach_nccl(self._h, buf, rank, world))

    @property
    def lora_world(self):
        return lib.pi05_lora_world(self._h)

    def lora_reset_optimizer(self):
        self._check(lib.pi05_lora_reset_optimizer(self._h))

    def lora_save_state(self, path):
        self._check(lib.pi05_lora_save_state(self._h, path.encode()))

    def lora_load_state(self, path):
        self._check(lib.pi05_lora_load_state(self._h, path.encode()))

    # -- reference-named extras
    def info(self):
        return {"kind": "pi05", "prefix_len": self.prefix_len, "max_batch": self.max_batch, **self.config.as_dict()}

    def set_stage(self, slot, stage, mode=1):
        self._check(lib.pi05_set_stage(self._h, slot, stage, mode))

    def set_act_config(self, act_dim=32, replan=16, mean=None, std=None, delta_mask=None, noise_seed=0):
        """pi05_set_act_config: output transform (z-score un-normalise, delta -> absolute actions on the
        dims of delta_mask, first act_dim dims) and re-plan period of act_batch / act."""
        keep = [None if v is None else np.ascontiguousarray(v, dt) for v, dt in
                ((mean, np.float32), (std, np.float32), (delta_mask, np.uint8))]
        c = ActConfig(act_dim, replan, *[None if k is None else k.ctypes.data for k in keep], noise_seed)
        self._check(lib.pi05_set_act_config(self._h, ctypes.byref(c)))
        self.act_dim = act_dim

    def set_noise_cholesky(self, L=None):
        """pi05_set_noise_cholesky: correlated re-plan noise L . eps (L lower-triangular [horizon*32]^2), None
        for uncorrelated noise"""
        if L is None:
            self._check(lib.pi05_set_noise_cholesky(self._h, None, 0))
            return
        Lc = np.ascontiguousarray(L, np.float32)
        self._check(lib.pi05_set_noise_cholesky(self._h, Lc.ctypes.data, Lc.shape[0]))

    def set_inpaint(self, fixed=0, t_min=0.3, corr=None):
        """pi05_set_inpaint: soft inpainting of the first `fixed` action rows after the steps that start above
        t_min, the rest corrected by corr [(horizon - fixed) * 32][fixed * 32]; fixed = 0 switches it off"""
        if not fixed:
            self._check(lib.pi05_set_inpaint(self._h, 0, float(t_min), None))
            return
        c = np.ascontiguousarray(corr, np.float32)
        H = self.config.horizon
        if c.shape != ((H - fixed) * 32, fixed * 32):
            raise ValueError(f"corr must be [{(H - fixed) * 32}][{fixed * 32}], got {c.shape}")
        self._check(lib.pi05_set_inpaint(self._h, int(fixed), float(t_min), c.ctypes.data))

    def set_kv_mix(self, wk=None, bk=None, wv=None, bv=None):
        """pi05_set_kv_mix: expert layer l attends to bf16(bf16(sum_j wk[l][j] K_j) + bk[l]) (V likewise);
        wk, wv [L][L], bk, bv [L][256]; no arguments switch mixing off"""
        if wk is None:
            self._check(lib.pi05_set_kv_mix(self._h, None, None, None, None))
            return
        L = self.config.gemma_layers
        arrs = [np.ascontiguousarray(a, np.float32) for a in (wk, bk, wv, bv)]
        for a, shape in zip(arrs, ((L, L), (L, 256), (L, L), (L, 256))):
            if a.shape != shape:
                raise ValueError(f"expected {shape}, got {a.shape}")
        self._check(lib.pi05_set_kv_mix(self._h, *[a.ctypes.data for a in arrs]))

    def set_inpaint_known(self, sample, known):
        """pi05_set_inpaint_known: the known rows [fixed][32] of batch position `sample`, None = free"""
        if known is None:
            self._check(lib.pi05_set_inpaint_known(self._h, int(sample), None))
            return
        k = np.ascontiguousarray(known, np.float32)
        self._check(lib.pi05_set_inpaint_known(self._h, int(sample), k.ctypes.data))

    @staticmethod
    def _frames(frames):
        """[n][n_cameras] frames (uint8 [h][w][3 or 4] numpy arrays or CUDA tensors, any row stride) ->
        (pi05_frame array, keep-alive list)"""
        flat, keep = [], []
        for row in frames:
            for f in row:
                if hasattr(f, "data_ptr"):  # torch tensor (host or CUDA), rows may be strided
                    h, w, c = f.shape
                    assert f.dtype.itemsize == 1 and f.stride(2) == 1 and f.stride(1) == c
                    flat.append(Frame(f.data_ptr(), h, w, c, f.stride(0)))
                else:
                    a = np.asarray(f)
                    if a.dtype != np.uint8 or a.strides[2] != 1 or a.strides[1] != a.shape[2]:
                        a = np.ascontiguousarray(a, np.uint8)
                    h, w, c = a.shape
                    flat.append(Frame(a.ctypes.data, h, w, c, a.strides[0]))
                keep.append(f if hasattr(f, "data_ptr") else a)
        arr = (Frame * len(flat))(*flat)
        return arr, keep

    def act_batch(self, slots, frames, tokens, state=None, noise=None, out=None):
        """pi05_act_batch: one receding-horizon step of the environment slots `slots`.  frames[i][c] is camera
        c of slot slots[i] at any size (RGB or RGBA, host or CUDA); tokens int32 [n][n_text]; state f32
        [n][act_dim] or None; noise f32 [n][horizon][32] or None (the slots' generator streams).  Returns
        f32 [n][act_dim] (or fills `out`, host or CUDA)."""
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        n = sl.shape[0]
        fa, fk = self._frames(frames)
        if out is None:
            out = np.empty((n, getattr(self, "act_dim", 32)), np.float32)
        pt, kt = _ptr(tokens, np.int32)
        ps, ks = _ptr(state, np.float32) if state is not None else (None, None)
        pz, kz = _ptr(noise, np.float32) if noise is not None else (None, None)
        po, ko = _ptr(out, np.float32, writable=True)
        self._check(lib.pi05_act_batch(self._h, n, sl.ctypes.data_as(ctypes.c_void_p), fa, pt, ps, pz, po))
        return out

    def act(self, slot, frames, tokens, state=None, noise=None):
        """pi05_act: act_batch for one slot; frames [n_cameras], tokens [n_text], state [act_dim],
        noise [horizon][32] or None.  Returns f32 [act_dim]."""
        fa, fk = self._frames([frames])
        out = np.empty((getattr(self, "act_dim", 32),), np.float32)
        pt, kt = _ptr(tokens, np.int32)
        ps, ks = _ptr(state, np.float32) if state is not None else (None, None)
        pz, kz = _ptr(noise, np.float32) if noise is not None else (None, None)
        self._check(lib.pi05_act(self._h, slot, fa, pt, ps, pz, out.ctypes.data))
        return out

    def reset_slot(self, slot):
        self._check(lib.pi05_reset_slot(self._h, slot))


class Tokenizer:
    """pi05_tokenizer: a SentencePiece BPE model file (identity normalization, byte fallback) and the
    pi0.5 prompt layout"""

    def __init__(self, model_path):
        err = ctypes.create_string_buffer(512)
        h = lib.pi05_tokenizer_load(model_path.encode(), err, len(err))
        if not h:
            raise Pi05Error(ERR_ARG, err.value.decode())
        self._h = ctypes.c_void_p(h)

    def close(self):
        if getattr(self, "_h", None):
            lib.pi05_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def vocab_size(self):
        return lib.pi05_tokenizer_vocab_size(self._h)

    def encode(self, text, add_bos=False):
        raw = text.encode()
        n = lib.pi05_tokenizer_encode(self._h, raw, int(add_bos), None, 0)
        if n < 0:
            raise Pi05Error(n, "pi05_tokenizer_encode")
        out = np.empty(max(n, 1), np.int32)
        lib.pi05_tokenizer_encode(self._h, raw, int(add_bos), out.ctypes.data, n)
        return out[:n].tolist()

    def prompt(self, task, state=None, max_len=200):
        """(ids int32 [max_len], mask bool [max_len]) of the pi0.5 prompt"""
        ids = np.empty(max_len, np.int32)
        mask = np.empty(max_len, np.uint8)
        st = None if state is None else np.ascontiguousarray(state, np.float32)
        n = lib.pi05_tokenize_prompt(self._h, task.encode(), None if st is None else st.ctypes.data,
                                     0 if st is None else st.size, max_len, ids.ctypes.data, mask.ctypes.data)
        if n < 0:
            raise Pi05Error(n, "pi05_tokenize_prompt")
        return ids, mask.astype(bool)


def read_weights_config(path):
    """pi05_read_weights_config: the Config a weight file's cfg lines describe (no GPU)"""
    c = Config()
    rc = lib.pi05_read_weights_config(path.encode(), ctypes.byref(c))
    if rc != OK:
        raise Pi05Error(rc, f"pi05_read_weights_config: cannot read {path}")
    return c


def create_batch(weights_path, device=0, max_batch=1):
    """pi05_create_batch (the reference's constructor): an Engine configured and loaded from the file"""
    h = lib.pi05_create_batch(weights_path.encode() if weights_path else None, device, max_batch)
    if not h:
        raise Pi05Error(ERR_ARG, f"pi05_create_batch failed for {weights_path}")
    eng = Engine.__new__(Engine)
    eng.config = read_weights_config(weights_path) if weights_path else Config.make()
    eng.max_batch = max_batch
    eng._h = ctypes.c_void_p(h)
    return eng


def nccl_unique_id():
    """pi05_nccl_unique_id: a new 128-byte NCCL id (rank 0 creates it and shares it with the others)"""
    buf = ctypes.create_string_buffer(128)
    rc = lib.pi05_nccl_unique_id(buf)
    if rc != OK:
        raise Pi05Error(rc, "pi05_nccl_unique_id: NCCL unavailable")
    return buf.raw


def resize_with_pad(image, out_h=224, out_w=224):
    """Camera frame (uint8 [h][w][3 or 4], any row stride) -> the zero-padded, aspect-preserving
    bilinear resize of pi05_resize_with_pad, uint8 [out_h][out_w][3].  Host only."""
    img = np.asarray(image)
    if img.dtype != np.uint8 or img.ndim != 3 or img.shape[2] not in (3, 4) or img.strides[1] != img.shape[2] \
            or img.strides[2] != 1:
        img = np.ascontiguousarray(img, dtype=np.uint8)
    h, w, c = img.shape
    out = np.empty((out_h, out_w, 3), np.uint8)
    rc = lib.pi05_resize_with_pad(img.ctypes.data_as(ctypes.c_void_p), h, w, c, img.strides[0],
                                  out.ctypes.data_as(ctypes.c_void_p), out_h, out_w)
    if rc != 0:
        raise Pi05Error(rc, f"pi05_resize_with_pad: unsupported frame {h}x{w}x{c} -> {out_h}x{out_w}")
    return out


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def normalize(x, a, b, mode="quantile", inverse=False):
    """pi05_normalize on a copy of x [..., dim]: mode "zscore" (a, b = mean, std) or "quantile"
    (a, b = q01, q99); inverse=True un-normalises."""
    y = _f32(x).copy()
    dim = y.shape[-1]
    av, bv = _f32(a), _f32(b)
    rc = lib.pi05_normalize(y.ctypes.data_as(ctypes.c_void_p), y.size // dim, dim, av.ctypes.data_as(ctypes.c_void_p),
                            bv.ctypes.data_as(ctypes.c_void_p), {"zscore": 0, "quantile": 1}[mode], int(inverse))
    if rc != 0:
        raise Pi05Error(rc, "pi05_normalize")
    return y


def discretize_state(x, bins=256):
    """pi05_discretize_state: int32 bins of a normalised state [..., dim]."""
    xv = _f32(x)
    out = np.empty(xv.shape, np.int32)
    dim = xv.shape[-1]
    rc = lib.pi05_discretize_state(xv.ctypes.data_as(ctypes.c_void_p), xv.size // dim, dim, bins,
                                   out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise Pi05Error(rc, "pi05_discretize_state")
    return out


def absolute_actions(actions, state, mask):
    """pi05_absolute_actions on a copy of actions [horizon][dim]: += state where mask."""
    y = _f32(actions).copy()
    st, mk = _f32(state), np.ascontiguousarray(mask, dtype=np.uint8)
    rc = lib.pi05_absolute_actions(y.ctypes.data_as(ctypes.c_void_p), y.shape[0], y.shape[1],
                                   st.ctypes.data_as(ctypes.c_void_p), mk.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise Pi05Error(rc, "pi05_absolute_actions")
    return y


def interp_actions_cubic(actions, n_out):
    """pi05_interp_actions_cubic: actions [n_in][dim] resampled to [n_out][dim] along a not-a-knot cubic spline."""
    a = _f32(actions)
    out = np.empty((n_out, a.shape[1]), np.float32)
    rc = lib.pi05_interp_actions_cubic(a.ctypes.data_as(ctypes.c_void_p), a.shape[0], a.shape[1],
                                       out.ctypes.data_as(ctypes.c_void_p), n_out)
    if rc != 0:
        raise Pi05Error(rc, "pi05_interp_actions_cubic")
    return out


def stage_vote(recent, current, max_stage=0):
    """pi05_stage_vote: the stage predicted twice among the last three of `recent`, else `current`."""
    r = np.ascontiguousarray(recent, dtype=np.int32)
    rc = lib.pi05_stage_vote(r.ctypes.data_as(ctypes.c_void_p), len(r), int(current), int(max_stage))
    if rc < 0:
        raise Pi05Error(rc, "pi05_stage_vote")
    return rc


def linear_static(x, w, out, bias=None, stream=None):
    """pi05_linear_static on CUDA bf16 tensors: out = x . w^T + bias with no device allocation.

    For callers that cannot allocate device memory; its scratch is a fixed 16 MiB device array
    inside the library, shared by all calls (calls that overlap on the GPU race).  `stream` is a
    raw cudaStream_t (int) or None for the legacy default stream.  Asynchronous.
    """
    T, K = x.shape
    F = w.shape[0]
    err = ctypes.create_string_buffer(512)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    rc = lib.pi05_linear_static(T, F, K, p(x), p(w), p(bias), p(out), ctypes.c_void_p(stream or 0), err, len(err))
    if rc != OK:
        raise Pi05Error(rc, err.value.decode())


def linear_static_status(stream=None):
    """pi05_linear_static_status: waits for `stream`; raises Pi05Error(ERR_DEVICE) if a
    pi05_linear_static call on the current device had a device-side wait give up."""
    err = ctypes.create_string_buffer(512)
    rc = lib.pi05_linear_static_status(ctypes.c_void_p(stream or 0), err, len(err))
    if rc != OK:
        raise Pi05Error(rc, err.value.decode())


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def synth_images(seed, sample, n_cameras=3):
    out = np.empty((n_cameras, 224, 224, 3), np.uint8)
    lib.pi05_synth_images(seed, sample, n_cameras, out.ctypes.data)
    return out


def synth_tokens(seed, sample, n_text=200):
    out = np.empty((n_text,), np.int32)
    lib.pi05_synth_tokens(seed, sample, n_text, out.ctypes.data)
    return out


def synth_noise(seed, sample, horizon=50):
    out = np.empty((horizon, 32), np.float32)
    lib.pi05_synth_noise(seed, sample, horizon, out.ctypes.data)
    return out


class Pi05NativePolicy:
    """Policy object in the place of the reference's glue/pi05_policy.py: forward(obs) -> action chunk.

    obs: {"images": uint8 [n][cams][224][224][3], "tokens": int32 [n][n_text], optional "noise"}.
    Returns fp32 [n][horizon][32].  Noise defaults to the seeded generator, one stream per call.
    """

    kind = "pi05"

    def __init__(self, engine, seed=0):
        self.engine = engine
        self.seed = seed
        self.calls = 0

    def forward(self, obs):
        imgs = obs["images"]
        n = imgs.shape[0]
        noise = obs.get("noise")
        if noise is None:
            noise = np.stack([synth_noise(self.seed, self.calls * 4096 + i, self.engine.config.horizon)
                              for i in range(n)])
        self.calls += 1
        return self.engine.infer(imgs, obs["tokens"], noise)

    def reset(self):
        self.calls = 0

    def set_stage(self, slot, stage, fixed=True):
        self.engine.set_stage(slot, stage, int(fixed))

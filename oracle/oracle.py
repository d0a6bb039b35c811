"""ctypes binding of the CPU oracle (oracle/libpi05_oracle.so).  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this module; the engine
never does.  The oracle is an fp32 restatement of the pi0.5 network (see pi05_oracle.cpp for the
reference citations).  Parity against the reference engine itself is unpinned: its source and its
golden dumps were deleted from the reference repository.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpi05_oracle.so")

# generator stream ids (behavior-2026_b200/csrc/pi05_model.h)
K_IN_IMAGE, K_IN_TOKENS, K_IN_NOISE, K_IN_KCACHE, K_IN_VCACHE, K_IN_ACTIONS, K_IN_TRAIN_NOISE = range(120, 127)
FP32_ACTIVATIONS = 1
TEXT_PAD_MASK = 2  # trailing prompt ids 0 are padding, masked as openpi masks it


def PREFIX_GROUP(g):
    """flags: prefix queries t < g attend to keys j < g only (two attention groups in the prefix)"""
    return int(g) << 16
HD = 256
GEM_W = 2048


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("siglip_layers", "gemma_layers", "expert_layers", "num_steps", "n_cameras", "n_text", "horizon")]

    @classmethod
    def make(cls, siglip_layers=27, gemma_layers=18, num_steps=10, n_cameras=3, n_text=200, horizon=50):
        return cls(siglip_layers, gemma_layers, gemma_layers, num_steps, n_cameras, n_text, horizon)

    @property
    def prefix_len(self):
        return 256 * self.n_cameras + self.n_text


PROBE = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64, ctypes.c_void_p)


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        cfg = P(Config)
        u8, i32, f32 = P(ctypes.c_uint8), P(ctypes.c_int32), P(ctypes.c_float)
        L.p5o_siglip.argtypes = [cfg, ctypes.c_uint64, u8, f32, ctypes.c_int, PROBE, ctypes.c_void_p]
        L.p5o_prefill.argtypes = [cfg, ctypes.c_uint64, u8, i32, f32, f32, ctypes.c_int, PROBE, ctypes.c_void_p]
        L.p5o_prefill_embedded.argtypes = [cfg, ctypes.c_uint64, f32, ctypes.c_int, f32, f32, ctypes.c_int, PROBE,
                                           ctypes.c_void_p]
        L.p5o_denoise.argtypes = [cfg, ctypes.c_uint64, f32, f32, ctypes.c_int, f32, f32, ctypes.c_int, PROBE,
                                  ctypes.c_void_p]
        L.p5o_denoise_inpaint.argtypes = [cfg, ctypes.c_uint64, f32, f32, ctypes.c_int, f32, f32, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_float, f32, f32]
        L.p5o_prefix_embed.argtypes = [cfg, ctypes.c_uint64, u8, i32, f32, ctypes.c_int]
        L.p5o_valid_prefix.argtypes = [cfg, i32, ctypes.c_int]
        L.p5o_gen_images.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, u8]
        L.p5o_gen_tokens.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, i32]
        L.p5o_gen_normal.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_double,
                                     ctypes.c_int, f32]
        L.p5o_gen_param.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_double, f32]
        L.p5o_gen_param_at.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_double, f32]
        for f in (L.p5o_gen_images, L.p5o_gen_tokens, L.p5o_gen_normal, L.p5o_gen_param, L.p5o_gen_param_at):
            f.restype = None
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


class Probe:
    """Collects named intermediate points (img.tokens, pre.l0.k, suf.s0.v, ...)."""

    def __init__(self, keep=None):
        self.keep = keep
        self.points = {}
        self._cb = PROBE(self._on)

    def _on(self, name, data, n, _ctx):
        name = name.decode()
        if self.keep is None or any(name.startswith(k) for k in self.keep):
            self.points[name] = np.ctypeslib.as_array(data, shape=(n,)).copy()


def _probe_args(probe):
    return (probe._cb if probe is not None else PROBE(), None)


# ---------------------------------------------------------------- synthetic workload
def gen_images(seed, sample, n_cam=3):
    out = np.empty((n_cam, 224, 224, 3), np.uint8)
    lib().p5o_gen_images(seed, sample, n_cam, _p(out, ctypes.c_uint8))
    return out


def gen_tokens(seed, sample, n=200):
    out = np.empty((n,), np.int32)
    lib().p5o_gen_tokens(seed, sample, n, _p(out, ctypes.c_int32))
    return out


def gen_normal(seed, kind, sub, shape, std=1.0, round_bf16=False):
    out = np.empty(shape, np.float32)
    lib().p5o_gen_normal(seed, kind, sub, out.size, std, int(round_bf16), _p(out, ctypes.c_float))
    return out


def gen_param(seed, kind, sub, shape, std=0.02):
    out = np.empty(shape, np.float32)
    lib().p5o_gen_param(seed, kind, sub, out.size, std, _p(out, ctypes.c_float))
    return out


def gen_param_at(seed, kind, sub, first, n, std=0.02):
    """elements [first, first + n) of a parameter stream"""
    out = np.empty((n,), np.float32)
    lib().p5o_gen_param_at(seed, kind, sub, first, n, std, _p(out, ctypes.c_float))
    return out


def gen_kv_cache(seed, sample, layers, P):
    """config-1 prefix cache: N(0,1) rounded to bf16, [layers][P][256] each for K and V."""
    k = gen_normal(seed, K_IN_KCACHE, sample, (layers, P, HD), 1.0, True)
    v = gen_normal(seed, K_IN_VCACHE, sample, (layers, P, HD), 1.0, True)
    return k, v


def gen_noise(seed, sample, horizon=50):
    return gen_normal(seed, K_IN_NOISE, sample, (horizon, 32), 1.0, False)


# ---------------------------------------------------------------- network
def siglip(cfg, seed, images, flags=0, probe=None):
    out = np.empty((256 * cfg.n_cameras, GEM_W), np.float32)
    images = np.ascontiguousarray(images, np.uint8)
    rc = lib().p5o_siglip(ctypes.byref(cfg), seed, _p(images, ctypes.c_uint8), _p(out, ctypes.c_float), flags,
                          *_probe_args(probe))
    assert rc == 0
    return out


def prefill(cfg, seed, images, tokens, flags=0, probe=None):
    P = cfg.prefix_len
    k = np.empty((cfg.gemma_layers, P, HD), np.float32)
    v = np.empty_like(k)
    images = np.ascontiguousarray(images, np.uint8)
    tokens = np.ascontiguousarray(tokens, np.int32)
    rc = lib().p5o_prefill(ctypes.byref(cfg), seed, _p(images, ctypes.c_uint8), _p(tokens, ctypes.c_int32),
                           _p(k, ctypes.c_float), _p(v, ctypes.c_float), flags, *_probe_args(probe))
    assert rc == 0
    return k, v


def prefix_embed(cfg, seed, images, tokens, flags=0):
    """SigLIP image tokens + scaled text embeddings, [P][2048] (bf16-valued floats)."""
    out = np.empty((cfg.prefix_len, GEM_W), np.float32)
    images = np.ascontiguousarray(images, np.uint8)
    tokens = np.ascontiguousarray(tokens, np.int32)
    rc = lib().p5o_prefix_embed(ctypes.byref(cfg), seed, _p(images, ctypes.c_uint8), _p(tokens, ctypes.c_int32),
                                _p(out, ctypes.c_float), flags)
    assert rc == 0
    return out


def prefill_embedded(cfg, seed, emb, flags=0, probe=None):
    emb = np.ascontiguousarray(emb, np.float32)
    P = emb.shape[0]
    k = np.empty((cfg.gemma_layers, P, HD), np.float32)
    v = np.empty_like(k)
    rc = lib().p5o_prefill_embedded(ctypes.byref(cfg), seed, _p(emb, ctypes.c_float), P, _p(k, ctypes.c_float),
                                    _p(v, ctypes.c_float), flags, *_probe_args(probe))
    assert rc == 0
    return k, v


def round_bf16(x):
    """float32 -> the nearest bf16 value (round to nearest, ties to even), as float32"""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).view(np.float32)


def kv_mix(cache, w, b):
    """KV layer mixing of the PiBehavior model (π05_네이티브엔진.md:140, a bf16 einsum over the prefix cache's
    layers plus a bf16 bias): out[l] = bf16(bf16(sum_j w[l][j] cache[j]) + b[l]) with w, b rounded to bf16,
    the sum in fp32 over j in order, each product and sum rounded (no contraction).  cache [L][P][256]."""
    cache = np.ascontiguousarray(cache, np.float32)
    w, b = round_bf16(np.asarray(w, np.float32)), round_bf16(np.asarray(b, np.float32))
    out = np.empty_like(cache)
    for l in range(cache.shape[0]):
        acc = np.zeros(cache.shape[1:], np.float32)
        for j in range(cache.shape[0]):
            acc = acc + np.float32(w[l, j]) * cache[j]
        out[l] = round_bf16(round_bf16(acc) + b[l][None, :])
    return out


def denoise(cfg, seed, kcache, vcache, noise, flags=0, probe=None, inpaint=None, mix=None):
    """inpaint = (known [fixed][32], corr [(horizon - fixed) * 32][fixed * 32], t_min): soft inpainting;
    mix = (wk, bk, wv, bv): the expert attends to the KV layer mixes of the prefix cache"""
    if mix is not None:
        wk, bk, wv, bv = mix
        kcache, vcache = kv_mix(kcache, wk, bk), kv_mix(vcache, wv, bv)
    kcache = np.ascontiguousarray(kcache, np.float32)
    vcache = np.ascontiguousarray(vcache, np.float32)
    noise = np.ascontiguousarray(noise, np.float32)
    P = kcache.shape[1]
    out = np.empty_like(noise)
    if inpaint is not None:
        assert probe is None
        known, corr, t_min = inpaint
        known = np.ascontiguousarray(known, np.float32)
        corr = np.ascontiguousarray(corr, np.float32)
        rc = lib().p5o_denoise_inpaint(ctypes.byref(cfg), seed, _p(kcache, ctypes.c_float),
                                       _p(vcache, ctypes.c_float), P, _p(noise, ctypes.c_float),
                                       _p(out, ctypes.c_float), flags, known.shape[0], t_min,
                                       _p(known, ctypes.c_float), _p(corr, ctypes.c_float))
        assert rc == 0
        return out
    rc = lib().p5o_denoise(ctypes.byref(cfg), seed, _p(kcache, ctypes.c_float), _p(vcache, ctypes.c_float), P,
                           _p(noise, ctypes.c_float), _p(out, ctypes.c_float), flags, *_probe_args(probe))
    assert rc == 0
    return out


def valid_prefix(cfg, tokens, flags=0):
    tokens = np.ascontiguousarray(tokens, np.int32)
    return lib().p5o_valid_prefix(ctypes.byref(cfg), _p(tokens, ctypes.c_int32), flags)


def infer(cfg, seed, images, tokens, noise, flags=0, probe=None, inpaint=None, mix=None):
    k, v = prefill(cfg, seed, images, tokens, flags, probe)
    s = valid_prefix(cfg, tokens, flags)  # with TEXT_PAD_MASK the padding's cache rows are left out
    return denoise(cfg, seed, k[:, :s], v[:, :s], noise, flags, probe, inpaint, mix)

"""CPU checks of the C ABI library: it loads, exports every symbol include/pi05.h declares, and its
host-side generators match the oracle's (no GPU compute is called here)."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "pi05.h")).read()
    return sorted(set(re.findall(r"PI05_API[^;(]*?\b(pi05_\w+)\s*\(", src)))


def test_header_declares_the_path(pn):
    syms = declared_symbols()
    for need in ("pi05_create", "pi05_load_weights", "pi05_prefill", "pi05_denoise", "pi05_infer",
                 "pi05_create_batch", "pi05_infer_batch", "pi05_set_stage"):
        assert need in syms


def test_library_exports_every_declared_symbol(pn):
    lib = ctypes.CDLL(pn.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(pn.EXPORTS) <= set(declared_symbols())


def test_default_config(pn):
    c = pn.Config()
    pn.lib.pi05_default_config(ctypes.byref(c))
    assert c.as_dict() == dict(siglip_layers=27, gemma_layers=18, expert_layers=18, num_steps=10, n_cameras=3,
                               n_text=200, horizon=50, batch_invariant=0, text_pad_mask=0, prefix_group=0)
    assert c.prefix_len == 968


def test_create_rejects_bad_config_without_gpu(pn):
    bad = pn.Config.make(gemma_layers=2)
    bad.expert_layers = 3  # expert layer l reads prefix layer l's cache: depths must match
    err = ctypes.create_string_buffer(256)
    assert not pn.lib.pi05_create(ctypes.byref(bad), 0, 1, err, 256)
    assert b"invalid configuration" in err.value


def test_synthetic_inputs_match_oracle_generator(pn, oracle):
    for s in (0, 3):
        assert np.array_equal(pn.synth_images(7, s), oracle.gen_images(7, s))
        assert np.array_equal(pn.synth_tokens(7, s), oracle.gen_tokens(7, s))
        assert np.array_equal(pn.synth_noise(7, s), oracle.gen_noise(7, s))
    tok = pn.synth_tokens(0, 0)
    assert tok.min() >= 0 and tok.max() < 257152


def test_bf16_helpers_round_to_nearest_even(pn):
    x = np.array([1.0, 1.00390625, 1.005859375, -0.1, 45.254833995939045], np.float32)
    bits = pn.f32_to_bf16_bits(x)
    back = pn.bf16_bits_to_f32(bits)
    # 1 + 2^-8 is a tie between 1 and 1+2^-7 -> even (1.0); 1.005859375 rounds up
    assert back.tolist() == [1.0, 1.0, 1.0078125, -0.10009765625, 45.25]


def test_lora_schedule_matches_optax_warmup_cosine(pn):
    """The reference recipe's schedule (openpi CosineDecaySchedule: optax warmup_cosine_decay_schedule with
    init lr / (warmup + 1)) restated in numpy, float64 rounded to float32; the default is constant."""
    import math

    c = pn.LoraConfig.reference_recipe()
    peak, end, w, d = float(np.float32(2.5e-5)), float(np.float32(2.5e-6)), 1000, 30000  # the struct holds float32

    def ref(k):
        if k < w:
            init = peak / (w + 1)
            return init + (peak - init) * k / w
        t = min(k - w, d - w)
        return end + (peak - end) * 0.5 * (1 + math.cos(math.pi * t / (d - w)))

    for k in (0, 1, 500, 999, 1000, 1001, 15000, 29999, 30000, 40000):
        assert pn.lora_schedule_lr(c, k) == np.float32(ref(k)), k
    flat = pn.LoraConfig()
    pn.lib.pi05_lora_default_config(ctypes.byref(flat))
    assert pn.lora_schedule_lr(flat, 0) == pn.lora_schedule_lr(flat, 5000) == np.float32(1e-4)


def test_engine_setters_reject_a_null_engine_without_gpu(pn):
    """The PiBehavior controls check their engine before touching the device."""
    z = np.zeros(16, np.float32)
    assert pn.lib.pi05_set_inpaint(None, 4, 0.3, z.ctypes.data) == -1
    assert pn.lib.pi05_set_inpaint_known(None, 0, z.ctypes.data) == -1
    assert pn.lib.pi05_set_kv_mix(None, z.ctypes.data, z.ctypes.data, z.ctypes.data, z.ctypes.data) == -1
    assert pn.lib.pi05_set_noise_cholesky(None, z.ctypes.data, 4) == -1
    assert pn.lib.pi05_prefill_embeds(None, 1, z.ctypes.data, z.ctypes.data) == -1

"""KV layer mixing (pi05_set_kv_mix, the PiBehavior model's expert reading a linear combination of the VLM
layers' K/V): expert layer l attends to bf16(bf16(sum_j w[l][j] K_j) + b[l]) and likewise for V.  The engine
against the oracle with the same mixing (oracle.kv_mix), on the same seeded weights and inputs.  Tolerance
(the parity contract): max-abs <= 2e-2 and cosine >= 0.999."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=3)


def cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def mixing(L, seed):
    """weights near 0.6 I with N(0, 0.1) spread, small biases; K and V differ"""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):
        w = (0.6 * np.eye(L) + rng.normal(0, 0.1, (L, L))).astype(np.float32)
        b = rng.normal(0, 0.05, (L, 256)).astype(np.float32)
        out += [w, b]
    return tuple(out)


def test_kv_mix_matches_oracle_reduced_depth(pn, oracle):
    """Full pipeline at reduced depth, batch of two; switching mixing off gives back the plain engine bit for
    bit."""
    cfg = pn.Config.make(**SMALL)
    eng = pn.Engine(cfg, max_batch=2)
    eng.init_random_weights(41)
    imgs = np.stack([pn.synth_images(42, i) for i in range(2)])
    toks = np.stack([pn.synth_tokens(42, i) for i in range(2)])
    noise = np.stack([pn.synth_noise(42, i) for i in range(2)])
    plain = eng.infer(imgs, toks, noise)
    mix = mixing(2, 43)
    eng.set_kv_mix(*mix)
    act = eng.infer(imgs, toks, noise)
    eng.set_kv_mix()
    np.testing.assert_array_equal(eng.infer(imgs, toks, noise), plain)
    eng.close()
    ocfg = oracle.Config.make(**SMALL)
    for i in range(2):
        ref = oracle.infer(ocfg, 41, imgs[i], toks[i], noise[i], mix=mix)
        d, c = float(np.abs(act[i] - ref).max()), cos(act[i], ref)
        print(f"reduced depth sample {i}: max-abs {d:.3e} cos {c:.6f}")
        assert d <= 2e-2 and c >= 0.999, (i, d, c)
        assert np.abs(act[i] - plain[i]).max() > 2e-2  # the mixing changes the chunk


def test_kv_mix_full_depth_denoise_matches_oracle(pn, oracle):
    """18-layer expert over an N(0,1) bf16 968-token prefix cache, 18 x 18 mixing of K and of V."""
    cfg = pn.Config.make()
    eng = pn.Engine(cfg, max_batch=1)
    eng.init_random_weights(0)
    eng.synth_prefix_cache(1, seed=0)
    mix = mixing(18, 44)
    eng.set_kv_mix(*mix)
    noise = pn.synth_noise(0, 0)
    act = eng.denoise(noise[None])[0]
    eng.close()
    k, v = oracle.gen_kv_cache(0, 0, 18, 968)
    ocfg = oracle.Config.make()
    ref = oracle.denoise(ocfg, 0, k, v, noise, mix=mix)
    d, c = float(np.abs(act - ref).max()), cos(act, ref)
    print(f"full depth: max-abs {d:.3e} cos {c:.6f}")
    assert d <= 2e-2 and c >= 0.999, (d, c)
    plain = oracle.denoise(ocfg, 0, k, v, noise)
    assert np.abs(plain - ref).max() > 2 * 2e-2  # through 18 layers the mixing moves the chunk a lot


def test_kv_mix_refusals(pn):
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=1)
    eng.init_random_weights(45)
    with pytest.raises(ValueError):
        eng.set_kv_mix(np.eye(3, dtype=np.float32), np.zeros((3, 256), np.float32), np.eye(3, dtype=np.float32),
                       np.zeros((3, 256), np.float32))
    eng.set_kv_mix(*mixing(2, 46))
    with pytest.raises(pn.Pi05Error, match="KV layer mixing"):
        eng.lora_init(seed=1, micro_batch=1)
    eng.close()

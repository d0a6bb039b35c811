"""CPU checks of the oracle: the conventions the reference engine's record pins, the committed golden
fixtures, and cross-checks of the C++ oracle against the independent torch restatements (vision tower:
oracle/siglip_ref.py; joint Gemma / expert network: oracle/lora_ref.py)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bf16(x):
    u = np.asarray([x], np.float32).view(np.uint32)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return float(u.astype(np.uint32).view(np.float32)[0])


def test_recorded_rounding_conventions():
    # Euler step multiplies v by dt rounded to bf16: bf16(-0.1) = -0.10009765625 (π05_네이티브엔진.md:39-40)
    assert bf16(-0.1) == -0.10009765625
    # Gemma embedder scale sqrt(2048) in the table dtype, SigLIP q divisor sqrt(72) in bf16
    assert bf16(np.sqrt(2048.0)) == 45.25
    assert bf16(np.sqrt(72.0)) == 8.5
    # flow-matching schedule t = 1, 0.9, ... accumulated in fp32 (openpi pi0.sample_actions)
    t, ts = np.float32(1.0), []
    for _ in range(10):
        ts.append(float(t))
        t = np.float32(t + np.float32(-0.1))
    assert ts[0] == 1.0 and abs(ts[-1] - 0.1) < 1e-6 and ts[1] == float(np.float32(0.9))


def test_generator_known_answers(oracle):
    kat = json.load(open(os.path.join(GOLDEN, "generator_kat.json")))
    assert oracle.gen_images(0, 0)[0, 0, :6].ravel()[:16].tolist() == kat["images_seed0_sample0_first16"]
    assert oracle.gen_tokens(0, 0)[:8].tolist() == kat["tokens_seed0_sample0_first8"]
    assert [float(x) for x in oracle.gen_noise(0, 0).ravel()[:8]] == kat["noise_seed0_sample0_first8"]
    assert [float(x) for x in oracle.gen_param(0, 32, 0, (8,))] == kat["gemma_wq_layer0_first8"]
    assert [float(x) for x in oracle.gen_param(0, 4, 0, (8,))] == kat["siglip_ln1_scale_layer0_first8"]


def test_generator_statistics(oracle):
    w = oracle.gen_param(0, 32, 0, (1 << 20,))
    assert abs(w.mean()) < 1e-4 and abs(w.std() - 0.02) < 2e-4
    ln = oracle.gen_param(0, 4, 0, (1 << 16,))  # LayerNorm scale = 1 + N(0, 0.02)
    assert abs(ln.mean() - 1.0) < 1e-3
    n = oracle.gen_noise(3, 1).ravel()
    assert abs(n.std() - 1.0) < 0.05
    tok = oracle.gen_tokens(0, 0, 4096)
    assert tok.min() >= 0 and tok.max() < 257152 and len(set(tok.tolist())) > 4000


def test_oracle_small_matches_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "oracle_small.npz"))
    cfg = oracle.Config.make(**json.loads(str(g["config"])))
    img = oracle.gen_images(11, 0, cfg.n_cameras)
    tok = oracle.gen_tokens(11, 0, cfg.n_text)
    noise = oracle.gen_noise(11, 0)
    act = oracle.infer(cfg, 11, img, tok, noise)
    np.testing.assert_allclose(act, g["actions"], rtol=0, atol=1e-6)
    # bf16 rounding points vs a pure-fp32 network: well inside the action tolerance
    assert np.abs(g["actions"] - g["actions_fp32"]).max() < 2e-2


def test_cpp_oracle_matches_torch_restatement(oracle):
    """Two independent restatements of the network agree: the first denoise velocity (t = 1, x_t = noise)
    of the C++ oracle and of the torch training forward with zero LoRA B (a plain network)."""
    import torch

    import lora_ref
    import siglip_ref

    cfg = oracle.Config.make(siglip_layers=1, gemma_layers=2, num_steps=10, n_cameras=1, n_text=16)
    img, tok, noise = oracle.gen_images(2, 0, 1), oracle.gen_tokens(2, 0, 16), oracle.gen_noise(2, 0)
    pr = oracle.Probe(keep=["suf.s0.v"])
    oracle.infer(cfg, 9, img, tok, noise, probe=pr)
    v_cpp = pr.points["suf.s0.v"].reshape(50, 32)
    nparam = sum(a * b for _, (a, b) in lora_ref.lora_layout(2))
    p = oracle.gen_normal(5, 80, 0, (nparam,), 0.01, True)
    ref = lora_ref.LoraRef(cfg, 9, p)
    for name, sl in ref.named_slices().items():  # zero every B: the adapters contribute nothing
        if name.endswith(".B"):
            with torch.no_grad():
                ref.params[name].zero_()
    emb = oracle.prefix_embed(cfg, 9, img, tok)[None]
    # the torch chain's own prefix (SigLIP restatement + Gemma embedder) gives the same embedding
    emb_t = siglip_ref.prefix_embedding(9, 1, img, tok)[None]
    assert np.abs(emb_t - emb).max() < 2e-2 * max(1.0, np.abs(emb).max())
    emb = emb_t
    with torch.no_grad():
        v_t = ref.velocity(emb, torch.from_numpy(noise[None]), np.array([1.0], np.float32))[0].numpy()
    assert np.abs(v_t - v_cpp).max() < 2e-2 and np.corrcoef(v_t.ravel(), v_cpp.ravel())[0, 1] > 0.9999


def test_cpp_oracle_siglip_matches_torch_restatement(oracle):
    """The vision tower (stem conv + learned posemb, pre-LN blocks, final LayerNorm, projector) of the C++
    oracle against the torch restatement written from flax's SigLIP modules, two layers, three cameras.
    Pure fp32 on both sides: max-abs <= 2e-2 (measured ~5e-4: fp32 summation order only, so a misplaced
    norm, a different GELU or posemb would show).  With bf16 activations the two round at slightly
    different points (the torch side also rounds the image, the conv output and the logits, as flax's
    bf16 modules do): every named point within rel-L2 2e-2."""
    import siglip_ref

    cfg = oracle.Config.make(siglip_layers=2, gemma_layers=1)
    img = oracle.gen_images(3, 0)
    ref32 = oracle.siglip(cfg, 7, img, flags=oracle.FP32_ACTIVATIONS)
    mine32 = siglip_ref.SiglipRef(2, 7, bf16=False)(img)
    assert np.abs(mine32 - ref32).max() <= 2e-2
    pr = oracle.Probe(keep=["img."])
    ref = oracle.siglip(cfg, 7, img, probe=pr)
    pts = {}
    mine = siglip_ref.SiglipRef(2, 7)(img, points=pts)
    pts["img.tokens"] = mine.ravel()
    pr.points["img.tokens"] = ref.ravel()
    for name in ("img.stem", "img.l0.out", "img.l1.out", "img.encoded", "img.tokens"):
        a, b = pts[name].astype(np.float64), pr.points[name].astype(np.float64)
        assert np.linalg.norm(a - b) / np.linalg.norm(b) <= 2e-2, name


def test_text_embedding_matches_oracle(oracle):
    """Gemma embedder rows x bf16(sqrt(2048)) of the torch restatement against the C++ oracle's txt.emb."""
    import siglip_ref

    cfg = oracle.Config.make(siglip_layers=0, gemma_layers=1, n_cameras=1, n_text=24)
    img, tok = oracle.gen_images(4, 0, 1), oracle.gen_tokens(4, 0, 24)
    emb = oracle.prefix_embed(cfg, 2, img, tok)[256:]
    np.testing.assert_array_equal(siglip_ref.text_embedding(2, tok), emb)


def test_oracle_inpaint_step_restates_the_formula(oracle):
    """Soft inpainting in the oracle, one Euler step (lands at t = 0): the first K values become the known
    actions and the rest move by corr . (x_K,new - x_K,old) from the free step; with t_min >= 1 no step
    qualifies and the result is the free denoise bit for bit."""
    cfg = oracle.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1, n_cameras=1, n_text=16)
    rng = np.random.default_rng(3)
    kc = rng.standard_normal((1, 40, 256)).astype(np.float32)
    vc = rng.standard_normal((1, 40, 256)).astype(np.float32)
    noise = oracle.gen_noise(4, 0)
    fixed, K = 4, 128
    known = rng.uniform(-1, 1, (fixed, 32)).astype(np.float32)
    corr = (rng.standard_normal((50 * 32 - K, K)) * 0.05).astype(np.float32)
    free = oracle.denoise(cfg, 5, kc, vc, noise)
    inp = oracle.denoise(cfg, 5, kc, vc, noise, inpaint=(known, corr, -1.0))
    np.testing.assert_array_equal(inp.ravel()[:K], known.ravel())
    delta = inp.ravel()[:K].astype(np.float32) - free.ravel()[:K].astype(np.float32)
    want = free.ravel()[K:] + (corr.astype(np.float64) @ delta.astype(np.float64)).astype(np.float32)
    np.testing.assert_allclose(inp.ravel()[K:], want, rtol=0, atol=1e-6)
    np.testing.assert_array_equal(oracle.denoise(cfg, 5, kc, vc, noise, inpaint=(known, corr, 1.0)), free)


def test_oracle_kv_mix(oracle):
    """The oracle's KV layer mixing: bf16 rounding equals torch's, identity weights with zero bias give the
    cache back, and a random mix is within two bf16 roundings of the float64 einsum."""
    import torch

    rng = np.random.default_rng(7)
    x = (rng.standard_normal(100000) * 10.0 ** rng.integers(-3, 4, 100000)).astype(np.float32)
    np.testing.assert_array_equal(oracle.round_bf16(x), torch.from_numpy(x).bfloat16().float().numpy())
    cache = oracle.round_bf16(rng.standard_normal((4, 30, 256)).astype(np.float32))
    np.testing.assert_array_equal(oracle.kv_mix(cache, np.eye(4), np.zeros((4, 256))), cache)
    w = oracle.round_bf16(rng.normal(0, 0.5, (4, 4)).astype(np.float32))
    b = oracle.round_bf16(rng.normal(0, 0.1, (4, 256)).astype(np.float32))
    want = np.einsum("lj,jpd->lpd", w.astype(np.float64), cache.astype(np.float64)) + b[:, None, :]
    got = oracle.kv_mix(cache, w, b)
    scale = np.einsum("lj,jpd->lpd", np.abs(w).astype(np.float64), np.abs(cache).astype(np.float64)) + np.abs(b)[:, None]
    assert (np.abs(got - want) <= 2 * 2.0 ** -8 * scale + 1e-30).all()

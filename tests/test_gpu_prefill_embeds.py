"""pi05_prefill_embeds: the text part of the prefix given as embeddings instead of token ids (for prompts that
are not sentences, as the PiBehavior model's task embeddings and stage tokens).  Given the engine's own text
embeddings of a prompt it reproduces the token path bit for bit; given other embeddings it matches the
oracle's prefill from the same embedding rows.  Tolerance (the parity contract): max-abs <= 2e-2 and
cosine >= 0.999."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=3)


def cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_prefill_embeds_of_the_prompt_equals_the_token_path(pn):
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=1)
    eng.init_random_weights(51)
    img, tok, noise = pn.synth_images(52, 0), pn.synth_tokens(52, 0), pn.synth_noise(52, 0)
    act, points = eng.verify(img[None], tok[None], noise[None], keep=["txt.emb"])
    emb = points["txt.emb"].reshape(1, 200, 2048)  # bf16 values as fp32: exact in bf16
    via_tokens = eng.infer(img[None], tok[None], noise[None])
    eng.prefill_embeds(img[None], emb)
    via_embeds = eng.denoise(noise[None])
    eng.close()
    np.testing.assert_array_equal(via_embeds, via_tokens)
    np.testing.assert_array_equal(via_tokens[0], act)


def test_prefill_embeds_matches_oracle(pn, oracle):
    """Batch of two with random (bf16) text rows, against the oracle's prefill from the same rows."""
    cfg = pn.Config.make(**SMALL)
    eng = pn.Engine(cfg, max_batch=2)
    eng.init_random_weights(53)
    rng = np.random.default_rng(54)
    imgs = np.stack([pn.synth_images(55, i) for i in range(2)])
    toks = np.stack([pn.synth_tokens(55, i) for i in range(2)])
    noise = np.stack([pn.synth_noise(55, i) for i in range(2)])
    emb = pn.bf16_bits_to_f32(pn.f32_to_bf16_bits(rng.normal(0, 1.0, (2, 200, 2048)).astype(np.float32)))
    eng.prefill_embeds(imgs, emb)
    act = eng.denoise(noise)
    with pytest.raises(ValueError):
        eng.prefill_embeds(imgs, emb[:, :100])
    eng.close()
    ocfg = oracle.Config.make(**SMALL)
    for i in range(2):
        full = oracle.prefix_embed(ocfg, 53, imgs[i], toks[i])
        full[768:] = emb[i]
        k, v = oracle.prefill_embedded(ocfg, 53, full)
        ref = oracle.denoise(ocfg, 53, k, v, noise[i])
        d, c = float(np.abs(act[i] - ref).max()), cos(act[i], ref)
        print(f"sample {i}: max-abs {d:.3e} cos {c:.6f}")
        assert d <= 2e-2 and c >= 0.999, (i, d, c)
        plain = oracle.infer(ocfg, 53, imgs[i], toks[i], noise[i])
        assert np.abs(act[i] - plain).max() > 2e-2  # the embeddings, not the tokens, made the prefix

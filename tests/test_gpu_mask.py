"""Prompts shorter than n_text (pi05_config.text_pad_mask = 1): the padding (ids 0) is masked as openpi
masks it -- no query attends to it and the action tokens' RoPE positions follow the last real token --
against the oracle with the same masking (oracle.TEXT_PAD_MASK), on the same seeded weights and inputs.
Tolerance (the parity contract): max-abs <= 2e-2 and cosine >= 0.999."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=3)


def cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def padded_inputs(pn, seed, lengths):
    imgs = np.stack([pn.synth_images(seed, i) for i in range(len(lengths))])
    toks = np.stack([pn.synth_tokens(seed, i) for i in range(len(lengths))])
    for i, n in enumerate(lengths):
        toks[i, n:] = 0
        toks[i, :n] = np.maximum(toks[i, :n], 1)  # real ids are never the padding id
    noise = np.stack([pn.synth_noise(seed, i) for i in range(len(lengths))])
    return imgs, toks, noise


@pytest.mark.parametrize("depth", ["small", "full"])
def test_masked_prompt_matches_oracle(pn, oracle, depth):
    kw = SMALL if depth == "small" else {}
    lengths = [37, 200, 120] if depth == "small" else [53]
    eng = pn.Engine(pn.Config.make(**kw, text_pad_mask=1), max_batch=len(lengths))
    eng.init_random_weights(17)
    imgs, toks, noise = padded_inputs(pn, 18, lengths)
    act = eng.infer(imgs, toks, noise)
    eng.close()
    ocfg = oracle.Config.make(**kw)
    for i, n in enumerate(lengths):
        ref = oracle.infer(ocfg, 17, imgs[i], toks[i], noise[i], flags=oracle.TEXT_PAD_MASK)
        d, c = float(np.abs(act[i] - ref).max()), cos(act[i], ref)
        print(f"{depth} length {n}: max-abs {d:.3e} cos {c:.6f}")
        assert d <= 2e-2 and c >= 0.999, (n, d, c)
        if n < 200:  # the mask moves the result by more than twice the tolerance: an unmasked engine fails
            plain = oracle.infer(ocfg, 17, imgs[i], toks[i], noise[i])
            assert np.abs(plain - ref).max() > 2 * 2e-2
            assert np.abs(act[i] - plain).max() > 2e-2


def test_masked_prompt_batch_invariant(pn):
    """Masking composes with batch invariance: every batch position equals its batch-of-one result."""
    eng = pn.Engine(pn.Config.make(**SMALL, text_pad_mask=1, batch_invariant=1), max_batch=3)
    eng.init_random_weights(19)
    imgs, toks, noise = padded_inputs(pn, 20, [90, 12, 200])
    batch = eng.infer(imgs, toks, noise)
    for i in range(3):
        np.testing.assert_array_equal(batch[i], eng.infer(imgs[i:i + 1], toks[i:i + 1], noise[i:i + 1])[0])
    eng.close()


def test_tokenized_prompt_through_act(pn, oracle, tmp_path):
    """A task string and a state, tokenized as openpi does (pi05_tokenize_prompt on a SentencePiece BPE model
    trained here), stepped through pi05_act_batch with the padding masked, against the oracle."""
    spm = pytest.importorskip("sentencepiece")
    text = tmp_path / "c.txt"
    rng = np.random.default_rng(21)
    words = "pick up the red cup turn on radio open drawer move left right Task State Action 0 1 2 3 4 5 6 7 8 9".split()
    text.write_text("\n".join(" ".join(rng.choice(words, 8)) for _ in range(2000)) + "\n")
    spm.SentencePieceTrainer.train(input=str(text), model_prefix=str(tmp_path / "m"), vocab_size=300, model_type="bpe",
                                   normalization_rule_name="identity", byte_fallback=True, add_dummy_prefix=False,
                                   remove_extra_whitespaces=False, split_digits=True, minloglevel=2)
    tok = pn.Tokenizer(str(tmp_path / "m.model"))
    state = rng.uniform(-1, 1, 23).astype(np.float32)
    ids, mask = tok.prompt("turn on the radio", state, 200)
    assert 20 < mask.sum() < 200 and not ids[mask.sum():].any()
    eng = pn.Engine(pn.Config.make(**SMALL, text_pad_mask=1), max_batch=1)
    eng.init_random_weights(22)
    eng.set_act_config(act_dim=32, replan=4)
    img, noise = pn.synth_images(23, 0), pn.synth_noise(23, 0)
    a = eng.act_batch([0], [[img[c] for c in range(3)]], ids[None], noise=noise[None])
    eng.close()
    ref = oracle.infer(oracle.Config.make(**SMALL), 22, img, ids, noise, flags=oracle.TEXT_PAD_MASK)
    assert np.abs(a[0] - ref[0]).max() <= 2e-2 and cos(a[0], ref[0]) >= 0.999


@pytest.mark.parametrize("depth,group", [("small", 769), ("small", 500), ("small", 768), ("full", 769)])
def test_prefix_groups_match_oracle(pn, oracle, depth, group):
    """Two attention groups in the prefix (pi05_config.prefix_group, the PiBehavior variant's image + base
    task block): prefix queries t < group attend to keys j < group only, on the tensor-core attention
    (per-row key limits, key splits that start past the group boundary) against the oracle with the same
    masking; 500 splits a 16-token query block, 768 ends on one.  Batch of two at reduced depth."""
    kw = SMALL if depth == "small" else {}
    n = 2 if depth == "small" else 1
    eng = pn.Engine(pn.Config.make(**kw, prefix_group=group), max_batch=n)
    eng.init_random_weights(27)
    imgs = np.stack([pn.synth_images(28, i) for i in range(n)])
    toks = np.stack([pn.synth_tokens(28, i) for i in range(n)])
    noise = np.stack([pn.synth_noise(28, i) for i in range(n)])
    act = eng.infer(imgs, toks, noise)
    eng.close()
    ocfg = oracle.Config.make(**kw)
    for i in range(n):
        ref = oracle.infer(ocfg, 27, imgs[i], toks[i], noise[i], flags=oracle.PREFIX_GROUP(group))
        d, c = float(np.abs(act[i] - ref).max()), cos(act[i], ref)
        print(f"{depth} group {group} sample {i}: max-abs {d:.3e} cos {c:.6f}")
        assert d <= 2e-2 and c >= 0.999, (group, i, d, c)
        if i == 0:
            plain = oracle.infer(ocfg, 27, imgs[i], toks[i], noise[i])
            # the engine is nearer the grouped oracle than the ungrouped one
            assert np.abs(act[i] - ref).max() < np.abs(act[i] - plain).max()
            if depth == "full":  # through 18 layers the groups move the chunk by more than twice the tolerance
                assert np.abs(plain - ref).max() > 2 * 2e-2
                assert np.abs(act[i] - plain).max() > 2e-2


def test_prefix_groups_refused_where_unsupported(pn):
    """The LoRA step trains one attention group; a group past the prefix is an invalid configuration."""
    eng = pn.Engine(pn.Config.make(**SMALL, prefix_group=769), max_batch=1)
    eng.init_random_weights(29)
    with pytest.raises(pn.Pi05Error, match="prefix_group"):
        eng.lora_init(seed=1, micro_batch=1)
    eng.close()
    with pytest.raises(pn.Pi05Error):
        pn.Engine(pn.Config.make(**SMALL, prefix_group=969), max_batch=1)

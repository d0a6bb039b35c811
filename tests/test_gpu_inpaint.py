"""Soft inpainting (pi05_set_inpaint / pi05_set_inpaint_known, the PiBehavior model's way of keeping a new
chunk continuous with the actions already committed): the first `fixed` action rows are put back on the
flow path of the known actions after every Euler step that starts above t_min, and the other rows follow
the Gaussian conditional through corr = Sigma_UO Sigma_OO^-1.  The engine against the oracle with the same
inpainting, on the same seeded weights and inputs.  Tolerance (the parity contract): max-abs <= 2e-2 and
cosine >= 0.999."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=10)
FIXED, T_MIN = 4, 0.3


def cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def correction(horizon, fixed, length=6.0):
    """Sigma_UO Sigma_OO^-1 of 0.5 I + 0.5 Sigma_t (the form of the record's noise covariance), Sigma_t
    smooth along the chunk (squared-exponential over the action index, independent action dimensions),
    in float64.  Its rows sum to at most 0.75 in absolute value, so the correction does not amplify the
    bf16-level difference of the known rows' update beyond the tolerance"""
    t = np.arange(horizon, dtype=np.float64)
    kt = 0.5 * np.exp(-0.5 * ((t[:, None] - t[None, :]) / length) ** 2) + 0.5 * np.eye(horizon)
    sigma = np.kron(kt, np.eye(32))
    K = fixed * 32
    return (sigma[K:, :K] @ np.linalg.inv(sigma[:K, :K])).astype(np.float32)


def inputs(pn, seed, n):
    imgs = np.stack([pn.synth_images(seed, i) for i in range(n)])
    toks = np.stack([pn.synth_tokens(seed, i) for i in range(n)])
    noise = np.stack([pn.synth_noise(seed, i) for i in range(n)])
    return imgs, toks, noise


def test_inpainting_matches_oracle(pn, oracle):
    """Batch of three: positions 0 and 1 inpainted towards different known rows, position 2 left free (it
    must match the plain oracle).  Switching inpainting off gives back the free engine bit for bit."""
    cfg = pn.Config.make(**SMALL)
    eng = pn.Engine(cfg, max_batch=3)
    eng.init_random_weights(31)
    imgs, toks, noise = inputs(pn, 32, 3)
    free = eng.infer(imgs, toks, noise)
    corr = correction(cfg.horizon, FIXED)
    rng = np.random.default_rng(33)
    known = rng.uniform(-1, 1, (2, FIXED, 32)).astype(np.float32)
    eng.set_inpaint(FIXED, T_MIN, corr)
    eng.set_inpaint_known(0, known[0])
    eng.set_inpaint_known(1, known[1])
    act = eng.infer(imgs, toks, noise)
    eng.set_inpaint(0)
    again = eng.infer(imgs, toks, noise)
    eng.close()
    np.testing.assert_array_equal(again, free)
    ocfg = oracle.Config.make(**SMALL)
    for i in range(3):
        ip = (known[i], corr, T_MIN) if i < 2 else None
        ref = oracle.infer(ocfg, 31, imgs[i], toks[i], noise[i], inpaint=ip)
        d, c = float(np.abs(act[i] - ref).max()), cos(act[i], ref)
        print(f"sample {i}: max-abs {d:.3e} cos {c:.6f}")
        assert d <= 2e-2 and c >= 0.999, (i, d, c)
        if i < 2:
            # the inpainting moves the chunk by more than twice the tolerance: an engine without it fails
            plain = oracle.infer(ocfg, 31, imgs[i], toks[i], noise[i])
            assert np.abs(plain - ref).max() > 2 * 2e-2
            assert np.abs(act[i] - plain).max() > 2e-2


def test_inpainting_known_rows_switch(pn):
    """A position switched back to free denoising (known = None) gives the free result bit for bit, and
    set_inpaint_known before set_inpaint is refused; bad shapes are refused."""
    cfg = pn.Config.make(**SMALL)
    eng = pn.Engine(cfg, max_batch=1)
    eng.init_random_weights(35)
    imgs, toks, noise = inputs(pn, 36, 1)
    with pytest.raises(pn.Pi05Error):
        eng.set_inpaint_known(0, np.zeros((FIXED, 32), np.float32))
    free = eng.infer(imgs, toks, noise)
    eng.set_inpaint(FIXED, T_MIN, correction(cfg.horizon, FIXED))
    np.testing.assert_array_equal(eng.infer(imgs, toks, noise), free)  # no position switched on yet
    eng.set_inpaint_known(0, np.full((FIXED, 32), 0.5, np.float32))
    assert np.abs(eng.infer(imgs, toks, noise) - free).max() > 2e-2
    eng.set_inpaint_known(0, None)
    np.testing.assert_array_equal(eng.infer(imgs, toks, noise), free)
    with pytest.raises(ValueError):
        eng.set_inpaint(FIXED, T_MIN, np.zeros((3, 3), np.float32))
    with pytest.raises(pn.Pi05Error):
        eng.set_inpaint(cfg.horizon, T_MIN, np.zeros((0, cfg.horizon * 32), np.float32))
    eng.close()

"""The reference's environment-step API through the C ABI: pi05_act_batch / pi05_act (camera frames as
the evaluator passes them, receding-horizon chunks, the wrapper's output transform) and bit-identical
batching (batch_invariant = 1), docs/archive/windows/π05_네이티브엔진.md:288-303.

Exact checks: camera frames of any size are resized on the GPU with pi05_resize_with_pad's arithmetic,
so an act step returns bit for bit the row that pi05_infer gives on the host-resized images of the same
batch; the output transform is compared bit for bit with its float32 numpy restatement; in the
batch-invariant mode pi05_act_batch equals stepping each slot alone with pi05_act, and pi05_infer at
any batch size equals batch-of-one calls, bit for bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=2)


def inputs(pn, seed, samples):
    return (np.stack([pn.synth_images(seed, i) for i in samples]), np.stack([pn.synth_tokens(seed, i) for i in samples]),
            np.stack([pn.synth_noise(seed, i) for i in samples]))


def frames224(images):
    """[n][cams][224][224][3] -> [n][cams] frames"""
    return [[images[i, c] for c in range(images.shape[1])] for i in range(images.shape[0])]


def test_act_batch_receding_horizon(pn):
    """A slot executes rows 0..replan-1 of the chunk pi05_infer gives for its inputs, then re-plans from
    the inputs of that call; pi05_reset_slot forces a re-plan; slots re-plan independently."""
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=2)
    eng.init_random_weights(8)
    replan, act_dim = 4, 23
    eng.set_act_config(act_dim=act_dim, replan=replan)
    im, tk, nz = inputs(pn, 1, [0, 1])
    ref = eng.infer(im, tk, nz)
    for step in range(replan):
        a = eng.act_batch([0, 1], frames224(im), tk, noise=nz)
        np.testing.assert_array_equal(a, ref[:, step, :act_dim])
    im2, tk2, nz2 = inputs(pn, 2, [0, 1])
    ref2 = eng.infer(im2, tk2, nz2)
    a = eng.act_batch([1, 0], frames224(im2[::-1]), tk2[::-1], noise=nz2[::-1])  # both re-plan
    np.testing.assert_array_equal(a, ref2[::-1, 0, :act_dim])
    eng.reset_slot(1)
    im3, tk3, nz3 = inputs(pn, 3, [0, 1])
    ref3 = eng.infer(im3[1:], tk3[1:], nz3[1:])
    a = eng.act_batch([0, 1], frames224(im3), tk3, noise=nz3)  # slot 0 continues, slot 1 re-plans
    np.testing.assert_array_equal(a[0], ref2[0, 1, :act_dim])
    np.testing.assert_array_equal(a[1], ref3[0, 0, :act_dim])
    eng.close()


def test_act_batch_frames_of_any_size_host_and_device(pn):
    """RGB / RGBA frames of several sizes with padded rows, in host memory and on the device, are
    resized on the GPU exactly as pi05_resize_with_pad resizes them on the host."""
    import torch

    rng = np.random.default_rng(5)
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=2)
    eng.init_random_weights(9)

    def host(h, w, c, pad=0):  # rows w * c + pad bytes apart
        buf = rng.integers(0, 256, (h, w * c + pad), dtype=np.uint8)
        return np.lib.stride_tricks.as_strided(buf, (h, w, c), (w * c + pad, c, 1))

    def dev(h, w, c, pad=0):
        t = torch.from_numpy(rng.integers(0, 256, (h, w * c + pad), dtype=np.uint8)).cuda()
        return t.as_strided((h, w, c), (w * c + pad, c, 1))

    frames = [[host(480, 640, 4, pad=12), dev(720, 720, 3), host(224, 224, 3)],
              [dev(300, 200, 3, pad=5), host(224, 300, 4), host(100, 120, 3, pad=1)]]
    imgs = np.stack([np.stack([pn.resize_with_pad(f.cpu().numpy() if hasattr(f, "cpu") else f) for f in row])
                     for row in frames])
    _, tk, nz = inputs(pn, 4, [0, 1])
    torch.cuda.synchronize()
    ref = eng.infer(imgs, tk, nz)
    eng.set_act_config(act_dim=32, replan=3)
    a = eng.act_batch([0, 1], frames, tk, noise=nz)
    np.testing.assert_array_equal(a, ref[:, 0, :])
    eng.close()


def test_act_output_transform_and_noise_stream(pn):
    """Un-normalise (z-score), add the state on the delta dims, keep act_dim dims: bit for bit the float32
    numpy restatement of openpi's Unnormalize + AbsoluteActions.  Without caller noise, a slot's first
    re-plan uses pi05_synth_noise(noise_seed, slot)."""
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=3)
    eng.init_random_weights(10)
    rng = np.random.default_rng(6)
    ad = 23
    mean = rng.normal(size=ad).astype(np.float32)
    std = rng.uniform(0.1, 2.0, size=ad).astype(np.float32)
    mask = (np.arange(ad) % 4 != 3).astype(np.uint8)
    eng.set_act_config(act_dim=ad, replan=2, mean=mean, std=std, delta_mask=mask, noise_seed=77)
    slots = [2, 0, 1]
    im, tk, _ = inputs(pn, 5, [0, 1, 2])
    nz = np.stack([pn.synth_noise(77, s) for s in slots])
    state = rng.normal(size=(3, ad)).astype(np.float32)
    raw = eng.infer(im, tk, nz)
    for step in range(2):
        a = eng.act_batch(slots, frames224(im), tk, state=state)
        r = raw[:, step, :ad] * (std + np.float32(1e-6)) + mean
        r = np.where(mask.astype(bool), r + state, r).astype(np.float32)
        np.testing.assert_array_equal(a, r)
    eng.close()


def test_act_batch_equals_act_bit_for_bit(pn):
    """batch_invariant = 1: four slots stepped together by pi05_act_batch (re-planning in batches of 1-4,
    generator noise) return, at every step, what each slot returns stepped alone with pi05_act
    (the reference's batch_test: 8 slots x 40 steps of act_batch against act, π05 record :303)."""
    cfg = pn.Config.make(**SMALL, batch_invariant=1)
    A = pn.Engine(cfg, max_batch=4)
    B = pn.Engine(cfg, max_batch=4)
    for e in (A, B):
        e.init_random_weights(11)
        e.set_act_config(act_dim=23, replan=3, noise_seed=3)
    for step in range(8):
        im, tk, _ = inputs(pn, 100 + step, range(4))
        if step == 4:
            A.reset_slot(2)
            B.reset_slot(2)
        slots = [0, 1, 2, 3] if step % 2 == 0 else [3, 1, 0, 2]
        idx = slots  # sample i of this step's inputs belongs to slot i
        a = A.act_batch(slots, frames224(im[idx]), tk[idx])
        for k, s in enumerate(slots):
            b = B.act(s, frames224(im[s:s + 1])[0], tk[s])
            np.testing.assert_array_equal(a[k], b, err_msg=f"step {step} slot {s}")
    A.close()
    B.close()


@pytest.mark.parametrize("depth,n", [("small", 16), ("full", 4)])
def test_batch_invariant_infer_equals_batch_of_one(pn, depth, n):
    """batch_invariant = 1: pi05_infer at batch n returns, for every sample, the bits a batch of one
    returns (the reference's batch path was bit-identical at n = 1/16/64/256, π05 record :299-302)."""
    kw = SMALL if depth == "small" else {}
    eng = pn.Engine(pn.Config.make(**kw, batch_invariant=1), max_batch=n)
    eng.init_random_weights(12)
    im, tk, nz = inputs(pn, 13, range(n))
    batch = eng.infer(im, tk, nz)
    for i in range(n):
        one = eng.infer(im[i:i + 1], tk[i:i + 1], nz[i:i + 1])[0]
        np.testing.assert_array_equal(batch[i], one, err_msg=f"sample {i}")
    eng.close()


def test_act_correlated_noise(pn):
    """pi05_set_noise_cholesky: without caller noise a re-plan draws L . eps (the PiBehavior model's
    N(0, 0.5 I + 0.5 Sigma) noise, fp64 accumulation on the device): the chunk equals pi05_infer's on the
    float64 numpy product rounded to float32, bit for bit; clearing L restores plain noise."""
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=2)
    eng.init_random_weights(14)
    eng.set_act_config(act_dim=32, replan=2, noise_seed=9)
    dim = 50 * 32
    rng = np.random.default_rng(15)
    a = rng.normal(size=(dim, dim)) / np.sqrt(dim)
    L = np.linalg.cholesky(0.5 * np.eye(dim) + 0.5 * (a @ a.T)).astype(np.float32)
    eng.set_noise_cholesky(L)
    im, tk, _ = inputs(pn, 16, [0, 1])
    eps = np.stack([pn.synth_noise(9, s) for s in (0, 1)]).reshape(2, dim)
    z = (L.astype(np.float64) @ eps.astype(np.float64).T).T.astype(np.float32).reshape(2, 50, 32)
    ref = eng.infer(im, tk, z)
    got = eng.act_batch([0, 1], frames224(im), tk)
    np.testing.assert_array_equal(got, ref[:, 0, :])
    eng.set_noise_cholesky(None)
    eng.reset_slot(0)
    eng.reset_slot(1)
    # second plan of each slot: elements [1600, 3200) of its stream, uncorrelated
    eps2 = np.stack([pn.synth_noise(9, s, horizon=100)[50:] for s in (0, 1)])
    ref2 = eng.infer(im, tk, eps2)
    np.testing.assert_array_equal(eng.act_batch([0, 1], frames224(im), tk), ref2[:, 0, :])
    eng.close()

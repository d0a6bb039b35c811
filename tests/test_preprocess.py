"""pi05_resize_with_pad (host camera-frame preprocessing) against Pillow.

The oracle is openpi's resize_with_pad geometry restated below over Pillow's own bilinear resize
(Pillow is test tooling here): aspect ratio kept, int() truncation of the resized size and of the
centring offsets, zero padding.  The library's port must match it bit for bit.  Runs on the CPU.
"""
import numpy as np
import pytest
from PIL import Image


def ref_resize_with_pad(img, out_h, out_w):
    rgb = np.ascontiguousarray(img[..., :3])
    h, w = rgb.shape[:2]
    if (h, w) == (out_h, out_w):
        return rgb.copy()
    ratio = max(w / out_w, h / out_h)
    rh, rw = int(h / ratio), int(w / ratio)
    resized = np.asarray(Image.fromarray(rgb).resize((rw, rh), resample=Image.BILINEAR))
    out = np.zeros((out_h, out_w, 3), np.uint8)
    ph, pw = max(0, int((out_h - rh) / 2)), max(0, int((out_w - rw) / 2))
    out[ph:ph + rh, pw:pw + rw] = resized
    return out


@pytest.mark.parametrize("h,w,c", [(480, 640, 3), (720, 1280, 4), (224, 224, 3), (100, 60, 3), (300, 224, 3),
                                   (37, 999, 3), (500, 501, 4), (223, 225, 3)])
def test_resize_with_pad_matches_pillow(pn, h, w, c):
    rng = np.random.default_rng(h * 1000 + w + c)
    img = rng.integers(0, 256, (h, w, c), dtype=np.uint8)
    got = pn.resize_with_pad(img)
    np.testing.assert_array_equal(got, ref_resize_with_pad(img, 224, 224))


def test_resize_with_pad_strided_rows_and_smooth_content(pn):
    """A frame that is a column window of a wider buffer (row stride > width x channels), with smooth
    content (gradients round differently from noise), and a non-square output."""
    rng = np.random.default_rng(7)
    yy, xx = np.mgrid[0:360, 0:700]
    base = np.stack([(xx * 255 // 699), (yy * 255 // 359), ((xx + yy) % 256)], -1).astype(np.uint8)
    base = np.concatenate([base, rng.integers(0, 256, (360, 700, 1), dtype=np.uint8)], -1)
    window = base[:, 40:680]  # strided view: rows 700 * 4 bytes apart
    assert window.strides[0] == 700 * 4
    got = pn.resize_with_pad(window, 192, 256)
    np.testing.assert_array_equal(got, ref_resize_with_pad(window, 192, 256))


def test_resize_with_pad_rejects_bad_frames(pn):
    with pytest.raises(pn.Pi05Error):
        pn.resize_with_pad(np.zeros((1, 4000, 3), np.uint8))  # resized height would be 0


# ---------------------------------------------------------------- state / action transforms
# numpy restatements of openpi's Normalize / Unnormalize (float32), the pi0.5 state discretisation
# (digitize over linspace(-1, 1, bins + 1)[:-1], minus one) and AbsoluteActions
def ref_normalize(x, a, b, mode, inverse):
    x, a, b = (np.asarray(v, np.float32) for v in (x, a, b))
    eps = np.float32(1e-6)
    if mode == "zscore":
        return x * (b + eps) + a if inverse else (x - a) / (b + eps)
    return (x + np.float32(1.0)) / np.float32(2.0) * (b - a + eps) + a if inverse else \
        (x - a) / (b - a + eps) * np.float32(2.0) - np.float32(1.0)


@pytest.mark.parametrize("mode", ["zscore", "quantile"])
@pytest.mark.parametrize("inverse", [False, True])
def test_normalize_matches_numpy(pn, mode, inverse):
    rng = np.random.default_rng(11)
    x = rng.normal(0, 3, (5, 23)).astype(np.float32)
    if mode == "zscore":
        a, b = rng.normal(0, 1, 23).astype(np.float32), rng.uniform(0.1, 2, 23).astype(np.float32)
    else:
        a = rng.uniform(-3, 0, 23).astype(np.float32)
        b = (a + rng.uniform(0.5, 4, 23)).astype(np.float32)
    np.testing.assert_array_equal(pn.normalize(x, a, b, mode, inverse), ref_normalize(x, a, b, mode, inverse))


def test_normalize_round_trip(pn):
    rng = np.random.default_rng(12)
    x = rng.uniform(-2, 2, (50, 32)).astype(np.float32)
    q01, q99 = np.full(32, -2.5, np.float32), np.full(32, 2.5, np.float32)
    y = pn.normalize(pn.normalize(x, q01, q99, "quantile"), q01, q99, "quantile", inverse=True)
    np.testing.assert_allclose(y, x, rtol=0, atol=2e-6)


def test_discretize_state_matches_numpy(pn):
    rng = np.random.default_rng(13)
    edges = np.linspace(-1, 1, 256 + 1)[:-1]
    x = np.concatenate([rng.uniform(-1.2, 1.2, (4, 23)).astype(np.float32).ravel(),
                        edges.astype(np.float32), np.float32([-1.0, 1.0, -1.0000001, 0.9921875, 0.99218744]),
                        np.float32([np.nan, -np.inf, np.inf])])
    x = x.reshape(-1, 1)  # every value, edges, the values just beside them, NaN and infinities included
    ref = (np.digitize(x, bins=edges) - 1).astype(np.int32)
    np.testing.assert_array_equal(pn.discretize_state(x, 256), ref)


def test_absolute_actions(pn):
    rng = np.random.default_rng(14)
    acts = rng.normal(size=(50, 23)).astype(np.float32)
    state = rng.normal(size=23).astype(np.float32)
    mask = (np.arange(23) % 3 != 2).astype(np.uint8)
    ref = acts.copy()
    ref[:, mask.astype(bool)] += state[mask.astype(bool)]
    np.testing.assert_array_equal(pn.absolute_actions(acts, state, mask), ref)


@pytest.mark.parametrize("n_in,n_out,dim", [(26, 20, 23), (4, 9, 3), (30, 26, 32), (12, 12, 5)])
def test_interp_actions_cubic_matches_scipy(pn, n_in, n_out, dim):
    """pi05_interp_actions_cubic against scipy interp1d(kind="cubic") (the not-a-knot spline) over the
    knots 0..n_in-1 sampled at n_out evenly spaced points of the same span; the engine solves in double
    precision and rounds once to float32."""
    interpolate = pytest.importorskip("scipy.interpolate")
    rng = np.random.default_rng(n_in * 100 + n_out)
    acts = np.cumsum(rng.normal(0, 0.1, (n_in, dim)), axis=0).astype(np.float32)
    ref = interpolate.interp1d(np.arange(n_in, dtype=np.float64), acts.astype(np.float64), kind="cubic",
                               axis=0)(np.linspace(0.0, n_in - 1.0, n_out))
    got = pn.interp_actions_cubic(acts, n_out)
    np.testing.assert_allclose(got, ref.astype(np.float32), rtol=0, atol=2e-6 * max(1.0, np.abs(ref).max()))
    np.testing.assert_array_equal(got[0], acts[0])  # the ends are knots
    np.testing.assert_allclose(got[-1], acts[-1], rtol=0, atol=1e-6)


def test_interp_actions_cubic_rejects_short_segments(pn):
    with pytest.raises(pn.Pi05Error):
        pn.interp_actions_cubic(np.zeros((3, 2), np.float32), 5)


def test_stage_vote(pn):
    assert pn.stage_vote([], 2) == 2
    assert pn.stage_vote([4], 2) == 2
    assert pn.stage_vote([4, 4], 2) == 4
    assert pn.stage_vote([1, 3, 3], 1) == 3
    assert pn.stage_vote([3, 1, 3], 1) == 3
    assert pn.stage_vote([5, 3, 1, 3], 1) == 3  # only the last three vote
    assert pn.stage_vote([0, 1, 2], 1) == 1  # no majority: stays
    assert pn.stage_vote([7, 7, 7], 0, max_stage=5) == 4  # capped below the task's stage count

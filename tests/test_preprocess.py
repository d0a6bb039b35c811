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

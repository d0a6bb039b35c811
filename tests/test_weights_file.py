"""Weight files (.pi05w) on the CPU: the manifest reader/writer, the engine -> reference layout
conversion, and pi05_read_weights_config through the C ABI (no GPU is used here)."""
import numpy as np


def test_pi05w_round_trip_bf16_and_f32(pn, tmp_path):
    import pi05w

    rng = np.random.default_rng(1)
    t = {"a.w": rng.normal(size=(3, 5)).astype(np.float32), "b": rng.normal(size=(7,)).astype(np.float32)}
    cfg = dict(siglip_layers=2, gemma_layers=3, expert_layers=3, num_steps=4, n_cameras=1, n_text=9, horizon=10)
    for dt in ("f32", "bf16"):
        path = str(tmp_path / f"x_{dt}.pi05w")
        pi05w.write(path, cfg, t, dt)
        c2, t2 = pi05w.read(path)
        assert c2 == cfg and set(t2) == set(t)
        for k in t:
            want = t[k] if dt == "f32" else pn.bf16_bits_to_f32(pn.f32_to_bf16_bits(t[k])).reshape(t[k].shape)
            np.testing.assert_array_equal(t2[k], want)
        c = pn.read_weights_config(path)
        assert c.as_dict() == dict(cfg, batch_invariant=0, text_pad_mask=0, prefix_group=0)


def test_reference_layout_conversion_shapes(pn):
    import pi05w

    cfg = dict(siglip_layers=1, gemma_layers=1, expert_layers=1, num_steps=1, n_cameras=1, n_text=1, horizon=50)
    rng = np.random.default_rng(2)
    eng = {"gem.l0.qkv.w": rng.normal(size=(2560, 8)).astype(np.float32),
           "gem.l0.gu.w": rng.normal(size=(6, 8)).astype(np.float32),
           "sig.l0.qkv.b": rng.normal(size=(1, 3456)).astype(np.float32),
           "sig.l0.mlp1.w": rng.normal(size=(4304, 4)).astype(np.float32),
           "sig.l0.mlp2.w": rng.normal(size=(4, 4304)).astype(np.float32),
           "sig.stem.w": rng.normal(size=(1152, 640)).astype(np.float32),
           "exp.ada.w": rng.normal(size=(3 * 3072, 2)).astype(np.float32)}
    ref = pi05w.to_reference_layout(cfg, eng)
    np.testing.assert_array_equal(ref["gem.l0.q.w"], eng["gem.l0.qkv.w"][:2048])
    np.testing.assert_array_equal(ref["gem.l0.v.w"], eng["gem.l0.qkv.w"][2304:])
    np.testing.assert_array_equal(ref["gem.l0.gate.w"], eng["gem.l0.gu.w"][0::2])
    np.testing.assert_array_equal(ref["gem.l0.up.w"], eng["gem.l0.gu.w"][1::2])
    assert ref["sig.l0.k.b"].shape == (1152,)
    assert ref["sig.l0.mlp1.w"].shape == (4352, 4) and not ref["sig.l0.mlp1.w"][4304:].any()
    assert ref["sig.l0.mlp2.w"].shape == (4, 4352) and not ref["sig.l0.mlp2.w"][:, 4304:].any()
    assert ref["sig.stem.w"].shape == (1152, 588)
    np.testing.assert_array_equal(ref["exp.l0.ada2.w"], eng["exp.ada.w"][3072:6144])
    np.testing.assert_array_equal(ref["exp.final.ada.w"], eng["exp.ada.w"][6144:])

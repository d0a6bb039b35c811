"""Weight files through the C ABI: pi05_save_weights -> pi05_load_weights, and the reference layout
written by behavior-2026_b200/pi05w.py (separate q/k/v and gate/up, SigLIP MLP padded to 4352, 588-column
patch embedding, per-norm modulation Denses, f32 or bf16) loaded by pi05_create_batch from the file's
cfg lines: the same chunks as the engine that produced the weights, bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(siglip_layers=1, gemma_layers=2, num_steps=2)


@pytest.fixture(scope="module")
def source(pn):
    eng = pn.Engine(pn.Config.make(**SMALL), max_batch=2)
    eng.init_random_weights(5)
    imgs = np.stack([pn.synth_images(6, i) for i in range(2)])
    toks = np.stack([pn.synth_tokens(6, i) for i in range(2)])
    noise = np.stack([pn.synth_noise(6, i) for i in range(2)])
    ref = eng.infer(imgs, toks, noise)
    yield eng, (imgs, toks, noise), ref
    eng.close()


def test_save_load_round_trip(pn, source, tmp_path):
    eng, batch, ref = source
    path = str(tmp_path / "engine.pi05w")
    eng.save_weights(path)
    other = pn.Engine(pn.Config.make(**SMALL), max_batch=2)
    other.init_random_weights(99)  # different weights first: the load must replace every tensor
    other.load_weights(path)
    np.testing.assert_array_equal(other.infer(*batch), ref)
    other.close()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_reference_layout_file_via_create_batch(pn, source, tmp_path, dtype):
    import pi05w

    eng, batch, ref = source
    path = str(tmp_path / f"ref_{dtype}.pi05w")
    pi05w.main(["--out", path, "--seed", "5", "--siglip-layers", "1", "--gemma-layers", "2", "--num-steps", "2",
                "--dtype", dtype])
    cfg, tensors = pi05w.read(path)
    assert "gem.l0.gate.w" in tensors and "gem.l0.qkv.w" not in tensors
    assert tensors["sig.l0.mlp1.w"].shape == (4352, 1152) and tensors["sig.stem.w"].shape == (1152, 588)
    e2 = pn.create_batch(path, 0, 2)
    assert e2.config.as_dict() == pn.Config.make(**SMALL).as_dict()
    np.testing.assert_array_equal(e2.infer_batch(*batch), ref)
    e2.close()


def test_load_refuses_mismatched_or_incomplete_files(pn, source, tmp_path):
    import pi05w

    eng, _, _ = source
    path = str(tmp_path / "w.pi05w")
    eng.save_weights(path)
    shallow = pn.Engine(pn.Config.make(siglip_layers=1, gemma_layers=1, num_steps=2), max_batch=1)
    with pytest.raises(pn.Pi05Error, match="gemma_layers 2 differs"):
        shallow.load_weights(path)
    shallow.close()
    cfg, tensors = pi05w.read(path)
    del tensors["exp.l1.down.w"]
    cut = str(tmp_path / "cut.pi05w")
    pi05w.write(cut, cfg, tensors, "bf16")
    other = pn.Engine(pn.Config.make(**SMALL), max_batch=1)
    with pytest.raises(pn.Pi05Error, match="exp.l1.down.w"):
        other.load_weights(cut)
    other.close()

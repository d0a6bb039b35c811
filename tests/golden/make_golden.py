"""Writes the golden fixtures of tests/golden/ from the CPU oracle.

The reference's own golden dumps for this path (data/pi05_native/ref*/*.pi05d, inputs_radio.npz,
docs/archive/windows/π05_네이티브엔진.md:46-51) are not in the reference checkout, so these fixtures pin
this repository's oracle instead: the seeded generator's first values (known-answer vectors) and the
action chunk of a small full-width configuration.  Regenerate with
    python tests/golden/make_golden.py
only when the oracle's arithmetic is meant to change.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402

SMALL = dict(siglip_layers=1, gemma_layers=1, num_steps=2, n_cameras=1, n_text=8, horizon=50)


def main():
    O.build()
    kat = {
        "images_seed0_sample0_first16": O.gen_images(0, 0)[0, 0, :6].ravel()[:16].tolist(),
        "tokens_seed0_sample0_first8": O.gen_tokens(0, 0)[:8].tolist(),
        "noise_seed0_sample0_first8": [float(x) for x in O.gen_noise(0, 0).ravel()[:8]],
        "gemma_wq_layer0_first8": [float(x) for x in O.gen_param(0, 32, 0, (8,))],
        "siglip_ln1_scale_layer0_first8": [float(x) for x in O.gen_param(0, 4, 0, (8,))],
    }
    with open(os.path.join(HERE, "generator_kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    cfg = O.Config.make(**SMALL)
    img = O.gen_images(11, 0, SMALL["n_cameras"])
    tok = O.gen_tokens(11, 0, SMALL["n_text"])
    noise = O.gen_noise(11, 0)
    act = O.infer(cfg, 11, img, tok, noise)
    act32 = O.infer(cfg, 11, img, tok, noise, flags=O.FP32_ACTIVATIONS)
    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), actions=act, actions_fp32=act32,
                        config=np.array(json.dumps(SMALL)))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()

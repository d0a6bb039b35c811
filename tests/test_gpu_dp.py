"""Data-parallel LoRA through the C ABI's own NCCL communicator (pi05_nccl_unique_id /
pi05_lora_attach_nccl): one process per GPU, the NCCL id handed from rank 0 over a gloo process group.

  * two ranks, each stepping its 2 samples with pi05_lora_step (per-layer gradient averages during the
    backward pass) end with bit-identical gradients and parameters, equal to those of
    pi05_lora_accumulate + pi05_lora_opt_step (whole-buffer average at the optimizer step); the averaged
    gradients match one GPU stepping all 4 samples within rel-L2 1e-2 and the loss within 1e-3 (a
    batch of 4 tiles the GEMMs differently from batches of 2, so activations round differently);
  * a communicator whose second rank never joins ends pi05_lora_attach_nccl with an error after
    PI05_NCCL_TIMEOUT_S instead of waiting for ever (the failure is made on the host; no kernel runs).
The two-rank case needs two GPUs and is skipped on one.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    import sys

    for p in (os.path.join(ROOT, "behavior-2026_b200"), os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _batch(pn, oracle, first, n):
    s = range(first, first + n)
    imgs = np.stack([pn.synth_images(21, i) for i in s])
    toks = np.stack([pn.synth_tokens(21, i) for i in s])
    acts = np.stack([oracle.gen_normal(21, oracle.K_IN_ACTIONS, i, (50, 32)) for i in s])
    noise = np.stack([oracle.gen_normal(21, oracle.K_IN_TRAIN_NOISE, i, (50, 32)) for i in s])
    t = np.linspace(0.1, 0.9, 4, dtype=np.float32)[first:first + n]
    return imgs, toks, acts, noise, t


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["PI05_NCCL_TIMEOUT_S"] = "60"
    _setup_paths()
    import torch.distributed as dist

    import dp
    import oracle
    import pi05native as pn

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        for mode in ("step", "accumulate"):
            eng = pn.Engine(pn.Config.make(siglip_layers=1, gemma_layers=2, num_steps=2), device=rank, max_batch=2)
            eng.init_random_weights(3)
            eng.lora_init(seed=4, micro_batch=2)
            dp.attach_nccl(eng, rank, world)
            b = _batch(pn, oracle, 2 * rank, 2)
            if mode == "step":
                out["loss"] = eng.lora_step(*b)
            else:
                eng.lora_zero_grads()
                eng.lora_accumulate(*b)
                eng.lora_opt_step()
            out[mode] = (eng.lora_get_params(), eng.lora_get_grads())
            out["world"] = eng.lora_world
            eng.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_two_rank_lora_step_over_the_engines_nccl(pn, oracle):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["world"] == 2
    for k in (0, 1):  # parameters, averaged gradients
        np.testing.assert_array_equal(res[0]["step"][k], res[1]["step"][k])
        np.testing.assert_array_equal(res[0]["step"][k], res[0]["accumulate"][k])
    assert res[0]["loss"] == res[1]["loss"]
    # one GPU, all four samples in one step
    eng = pn.Engine(pn.Config.make(siglip_layers=1, gemma_layers=2, num_steps=2), max_batch=4)
    eng.init_random_weights(3)
    eng.lora_init(seed=4, micro_batch=4)
    loss1 = eng.lora_step(*_batch(pn, oracle, 0, 4))
    g1 = eng.lora_get_grads().astype(np.float64)
    eng.close()
    g2 = res[0]["step"][1].astype(np.float64)
    assert np.linalg.norm(g2 - g1) / np.linalg.norm(g1) <= 1e-2
    assert abs(res[0]["loss"] - loss1) <= 1e-3 * abs(loss1)


@pytest.mark.timeout(300)
def test_attach_gives_up_when_a_rank_never_joins(pn, monkeypatch):
    monkeypatch.setenv("PI05_NCCL_TIMEOUT_S", "5")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    eng = pn.Engine(pn.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1), max_batch=1)
    eng.init_random_weights(1)
    eng.lora_init(seed=2, micro_batch=1)
    with pytest.raises(pn.Pi05Error, match="timed out"):
        eng.lora_attach_nccl(pn.nccl_unique_id(), 0, 2)  # rank 1 of 2 never joins
    assert eng.lora_world == 1
    eng.close()

"""Host-side multi-rank logic on CPU with gloo ranks (world size 2): batch sharding, the gradient
average that the LoRA step applies between accumulate and the optimizer step, and the hand-over of the
NCCL id with which every rank attaches its engine's own communicator."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "behavior-2026_b200"))
    import dp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        first, count = dp.shard(64, world, rank)
        # each rank's "gradient" = its rank-specific contribution; the average is known in closed form
        g = torch.arange(10, dtype=torch.float32) * (rank + 1)
        dp.allreduce_mean_(g, world)
        # the NCCL id of the engine's communicator travels from rank 0 over the process group
        import pi05native as pn
        uid = dp.exchange_unique_id(pn.nccl_unique_id() if rank == 0 else None, rank)
        q.put((rank, first, count, g.tolist(), uid))
    finally:
        dist.destroy_process_group()


def test_shard_and_gradient_average_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, f0, c0, g0, u0), (r1, f1, c1, g1, u1) = out
    assert (f0, c0, f1, c1) == (0, 32, 32, 32)
    assert isinstance(u0, bytes) and len(u0) == 128 and u0 == u1
    expect = [i * 1.5 for i in range(10)]  # mean of i*1 and i*2
    assert g0 == pytest.approx(expect) and g1 == pytest.approx(expect)


def test_shard_rejects_uneven_split():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "behavior-2026_b200"))
    import dp

    assert dp.shard(64, 8, 7) == (56, 8)
    with pytest.raises(ValueError):
        dp.shard(64, 3, 0)

"""Data parallelism for the pi0.5 engine: batch sharding and the LoRA gradient exchange.

The reference engine was single-GPU (docs/archive/windows/π05_네이티브엔진.md:464).  Here:
  * inference shards independent environments across ranks with no collective (`shard`);
  * the LoRA step averages the flat fp32 adapter-gradient buffer (26.5 M floats at full depth) over
    the ranks.  `attach_nccl` gives the engine its own NCCL communicator (pi05_lora_attach_nccl): the
    engine then averages each layer's gradients during the backward pass, on its own stream, inside
    pi05_lora_step.  torch.distributed only carries the 128-byte NCCL id from rank 0 to the others.
    `lora_allreduce` is the host-ordered alternative through torch.distributed (any backend).
One process per GPU.
"""
import torch


def exchange_unique_id(uid, rank):
    """rank 0's 128-byte id to every rank over the default process group (any backend)"""
    import torch.distributed as dist

    box = [uid if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def attach_nccl(engine, rank, world):
    """make `engine` (after lora_init) a member of a `world`-rank NCCL communicator; no-op for one rank"""
    if world == 1:
        return
    import pi05native as pn

    uid = exchange_unique_id(pn.nccl_unique_id() if rank == 0 else None, rank)
    engine.lora_attach_nccl(uid, rank, world)


def shard(n_global, world, rank):
    """(first sample, count) of `rank`'s share of `n_global` independent samples (contiguous blocks)."""
    if n_global % world:
        raise ValueError(f"{n_global} samples do not split over {world} ranks")
    per = n_global // world
    return rank * per, per


class _DeviceBuffer:
    """zero-copy view of an engine-owned device buffer for torch (CUDA array interface)"""

    def __init__(self, ptr, n, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def grad_tensor(engine):
    """the engine's flat LoRA gradient buffer as a CUDA torch tensor (no copy)"""
    return torch.as_tensor(_DeviceBuffer(engine.lora_grad_ptr(), engine.lora_num_params), device="cuda")


def allreduce_mean_(t, world):
    """in place: t <- mean over ranks of t (sum allreduce, then / world)"""
    if world == 1:
        return t
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    t.div_(world)
    return t


def lora_allreduce(engine, world):
    """average the accumulated LoRA gradients over ranks; orders the engine stream around the collective"""
    if world == 1:
        return
    engine.sync()  # gradients complete on the engine stream
    allreduce_mean_(grad_tensor(engine), world)
    torch.cuda.synchronize()  # collective complete before the optimizer reads the buffer

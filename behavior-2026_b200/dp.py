"""Data parallelism for the pi0.5 engine: batch sharding and the LoRA gradient allreduce.

The reference engine was single-GPU (docs/archive/windows/π05_네이티브엔진.md:464).  Here:
  * inference shards independent environments across ranks with no collective (`shard`);
  * the LoRA step allreduces the flat fp32 adapter-gradient buffer (26.5 M floats at full depth)
    between pi05_lora_accumulate and pi05_lora_opt_step, averaging over ranks (`allreduce_mean_`).
One process per GPU; torch.distributed supplies the communicator (NCCL on GPUs, gloo on CPU).
"""
import torch


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

"""One-process-per-GPU plumbing for the sharded path (torch.distributed).

Every BASELINE config splits into independent contiguous shards -- element
ranges for maps, row ranges for softmax and GEMM M-blocks, batch ranges for
the scaled-scores softmax -- so no data-path collective exists. The only
collective is the optional all-gather that assembles a sharded result on
every rank (NCCL over NVLink), used when a caller wants the whole result on
one device. The reference has no distributed layer at all (it is a single
process, single device executor); this module is new.
"""
from __future__ import annotations

import datetime
import os


def shard(units: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced shard [begin, end) of `units` for `rank`; the
    same split the C++ host entry uses for in-process multi-GPU runs."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return units * rank // world, units * (rank + 1) // world


def env_rank() -> tuple[int, int, int]:
    """(world, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, local_rank: int, timeout_s: float = 120.0):
    """Initialise the default process group with a short timeout, so ranks
    that wait for a rank that died end with an error instead of hanging."""
    import torch
    import torch.distributed as dist

    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(backend, **kwargs)
    return dist


def max_over_ranks(value: float, dist, device=None) -> float:
    """The maximum of a per-rank scalar (e.g. a kernel time) over all ranks."""
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_gather_shards(local, dist):
    """All-gather equal-sized contiguous shards into the full result on every
    rank (NCCL all_gather_into_tensor over NVLink for CUDA tensors)."""
    import torch

    world = dist.get_world_size()
    out = torch.empty((world * local.numel(),), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.reshape(-1).contiguous())
    return out

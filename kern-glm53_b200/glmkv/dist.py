"""Process-per-GPU plumbing for the layer-group stages (torch.distributed; NCCL on GPUs, gloo on CPU).

The cache path itself has no collective: each rank owns whole layers. These helpers only place the
stages and combine timings: the slowest rank's time is the job's (every rank takes the same
collective steps in the same order, so a rank that fails or leaves makes the others' next collective
end with an error after the process group's timeout instead of hanging).
"""
import datetime
import os

import torch
import torch.distributed as dist

from . import stage


def env():
    """(world, rank, local_rank) from the torchrun environment (1, 0, 0 without it)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend, timeout_s=300, device=None):
    """Join the process group when there is more than one rank; returns (world, rank, local_rank)."""
    world, rank, local = env()
    if world > 1 and not dist.is_initialized():
        kw = {"device_id": device} if device is not None and backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local


def assignment(world, **kw):
    """[(first, last)] layer range of every rank: stage cuts at indexer layers, balanced by bytes."""
    c = list(stage.cuts(world, **kw)) + [stage.LAYERS]
    return [(c[i], c[i + 1]) for i in range(world)]


def max_over_ranks(value, device=None):
    """The largest `value` over all ranks (the value itself with one rank)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, device=None):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_objects(obj):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def barrier():
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def finish():
    if dist.is_initialized():
        dist.destroy_process_group()

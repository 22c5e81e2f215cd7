"""Host-side helpers for running seal/open on several GPUs of one node.

KV objects are independent, so each GPU (one process per GPU) seals and opens
its own objects with its own key handle and stream; no data crosses between
GPUs. torch.distributed is used only for the timing barrier and to take the
max of per-rank device times (the job takes as long as its slowest GPU).
"""

from __future__ import annotations

import os


def rank_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def round_robin(num_objects: int, rank: int, world: int) -> list[int]:
    """Indices of the objects rank `rank` of `world` processes owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return list(range(rank, num_objects, world))


def kv_head_shard(heads: int, rank: int, world: int) -> range:
    """KV heads of a tensor-parallel rank (contiguous block of heads/world)."""
    if heads % world:
        raise ValueError("heads must divide evenly across ranks")
    per = heads // world
    return range(rank * per, (rank + 1) * per)


def reduce_max(values, device=None) -> list[float]:
    """Element-wise max over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    vals = [float(v) for v in values]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.cpu().tolist()


def reduce_sum(values, device=None) -> list[float]:
    """Element-wise sum over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    vals = [float(v) for v in values]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().tolist()


def all_ok(flag: bool, device=None) -> bool:
    """True only if every rank passes True."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return bool(flag)
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())

"""Head sharding of the Spark layer across the GPUs of one node.

Every stage of the layer (pooling, routing, Top-K, summaries, reblock, attention) is
independent per (batch, head), so N ranks each take a contiguous range of heads and run the
layer on it with no data-path exchange.  The only collective is the timing reduction (the
slowest rank defines the job's time).  Works with any torch.distributed backend: NCCL on the
GPUs, gloo on CPU for the tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_shard(heads: int, world: int, rank: int) -> slice:
    """Contiguous heads of `rank`; heads must divide evenly so every rank does equal work."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly across {world} ranks")
    per = heads // world
    return slice(rank * per, (rank + 1) * per)


def shard_heads(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's heads of a BTHD tensor, contiguous."""
    return x[:, :, head_shard(x.shape[2], world, rank)].contiguous()


def max_over_ranks(values, device=None) -> list[float]:
    """Element-wise maximum of per-rank floats (times) across the process group; identity
    without one.  Every rank must call it with the same number of values."""
    values = [float(v) for v in values]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return values
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]

"""The multi-GPU path's host logic on CPU: two gloo ranks shard the heads, run a per-head
computation on their shard with no exchange, and reduce their times to the maximum, as
bench.py does over NCCL.  A rank that fails before the collective makes the other rank's
collective end with an error instead of waiting for good."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spark_h3_b200.sharding import head_shard, max_over_ranks, shard_heads


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def per_head_work(x: torch.Tensor) -> torch.Tensor:
    """A stand-in for the layer: independent per (batch, head)."""
    return torch.softmax(x @ x.transpose(-1, -2), dim=-1) @ x


def _worker(rank, world, port, results, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, 16, 8, 4, generator=g)  # B, T, H, D
        local = shard_heads(x, world, rank)
        out = per_head_work(local.permute(0, 2, 1, 3)).permute(0, 2, 1, 3)
        if rank == fail_rank:
            raise RuntimeError("planted failure")
        times = max_over_ranks([1.0 + rank, 10.0 - rank])
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        results[rank] = dict(times=times, out=torch.cat(gathered, dim=2), shard=head_shard(8, world, rank))
    except Exception as err:  # noqa: BLE001 - the parent inspects what each rank saw
        results[rank] = dict(error=f"{type(err).__name__}: {err}")
    finally:
        dist.destroy_process_group()


def run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, free_port_cache[0], results, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish")
    return dict(results)


free_port_cache = [0]


def test_two_ranks_shard_heads_and_reduce_times():
    free_port_cache[0] = free_port()
    res = run(2)
    x = torch.randn(1, 16, 8, 4, generator=torch.Generator().manual_seed(0))
    expected = per_head_work(x.permute(0, 2, 1, 3)).permute(0, 2, 1, 3)
    for rank in range(2):
        assert "error" not in res[rank], res[rank]
        assert res[rank]["times"] == [2.0, 10.0]
        assert torch.allclose(res[rank]["out"], expected, atol=1e-6)
    assert res[0]["shard"] == slice(0, 4) and res[1]["shard"] == slice(4, 8)


def test_failed_rank_ends_the_collective_with_an_error():
    free_port_cache[0] = free_port()
    res = run(2, fail_rank=1)
    assert "planted failure" in res[1]["error"]
    assert "error" in res[0]  # its all_reduce ended (peer gone or timeout), it did not hang


def test_uneven_split_rejected():
    with pytest.raises(ValueError, match="split evenly"):
        head_shard(32, 3, 0)
    assert max_over_ranks([3.0, 1.5]) == [3.0, 1.5]

"""Config-4 DiT block stack: the sequence <-> head exchange on two gloo ranks (CPU), and on
the GPU one block stack step against an fp32 restatement of the same block math."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from spark_h3_b200.dit import (DiTConfig, DiTStack, exchange_to_heads, exchange_to_tokens, reference_block_math,
                               rope_tables, token_coords)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        nloc, H, D = 3, 4, 2
        hp = H // world
        # value = global token * 100 + head * 10 + dim
        tok = torch.arange(rank * nloc, (rank + 1) * nloc).view(nloc, 1, 1)
        head = torch.arange(H).view(1, H, 1)
        dim = torch.arange(D).view(1, 1, D)
        local = (tok * 100 + head * 10 + dim).float()  # [Nloc, H, D]
        send = local.view(nloc, world, hp, D).permute(1, 0, 2, 3).contiguous()  # the kernel's send layout
        heads = exchange_to_heads(send)  # [N, Hp, D]
        back = exchange_to_tokens(heads, world)  # [P, Nloc, Hp, D]
        results[rank] = dict(heads=heads, back=back, local=local)
    except Exception as err:  # noqa: BLE001
        results[rank] = dict(error=repr(err))
    finally:
        dist.destroy_process_group()


def test_exchange_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    for rank in range(2):
        r = results[rank]
        assert "error" not in r, r
        N, hp = 6, 2
        expected = torch.stack([torch.stack([torch.tensor([t * 100 + (rank * hp + h) * 10 + d for d in range(2)])
                                             for h in range(hp)]) for t in range(N)]).float()
        assert torch.equal(r["heads"], expected)
        # back to this rank's tokens: segment p holds the heads of rank p
        seg = r["back"].permute(1, 0, 2, 3).reshape(3, 4, 2)
        assert torch.equal(seg, r["local"])


def test_rope_tables_and_coords():
    cfg = DiTConfig()
    inv, axis = rope_tables(cfg, "cpu")
    assert inv.shape == (64,) and axis.tolist() == [0] * 16 + [1] * 24 + [2] * 24
    assert inv[0] == 1.0 and inv[15] < inv[14]
    c = token_coords((3, 4, 5), 7, 5, "cpu")
    assert c.tolist() == [[0, 1, 2], [0, 1, 3], [0, 1, 4], [0, 2, 0], [0, 2, 1]]


@pytest.mark.gpu
@pytest.mark.parametrize("dense", [True, False])
def test_stack_step_matches_block_math(cuda_device, dense):
    cfg = DiTConfig(hidden=256, heads=2, ffn=512, blocks=2)
    grid = (2, 16, 32)
    stack = DiTStack(cfg, grid, device=cuda_device, seed=3, spark_mode="reweight_only", topk_ratio=0.2)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    x0 = torch.randn(stack.local, cfg.hidden, device=cuda_device, generator=g).to(torch.bfloat16)
    x = stack.step(x0.clone(), 500.0, dense=dense)

    def attention(q, k, v):
        if dense:
            o = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                               v.float().transpose(1, 2))
            return o.transpose(1, 2).to(torch.bfloat16)
        from spark_h3_b200.attention import spark_attention_bthd

        return spark_attention_bthd(stack.controller, q.contiguous(), k.contiguous(), v.contiguous(), stack.layout, 0)

    ref = x0
    for blk, mod in zip(stack.blocks, stack.modulation(500.0)):
        ref = reference_block_math(ref, blk, mod, cfg, stack.coords, stack.inv_freq, stack.axis, attention)
    diff = (x.float() - ref.float()).abs().max().item()
    cos = F.cosine_similarity(x.float().flatten(), ref.float().flatten(), dim=0).item()
    assert torch.isfinite(x).all()
    assert cos > 0.999 and diff <= 0.05 * ref.float().abs().max().item(), (cos, diff)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2])
def test_fused_producer_matches_separate_path(cuda_device, world):
    """sb_fp8_gemm_qkv_rope (norm and RoPE in the GEMM epilogue) against sb_fp8_gemm +
    sb_dit_qkv_norm_rope, in the send layout of `world` shards."""
    from spark_h3_b200.dit import DiTConfig, DiTStack

    cfg = DiTConfig(hidden=512, heads=4, ffn=1024, blocks=1)
    grid = (2, 16, 24)
    stack = DiTStack(cfg, grid, device=cuda_device, world=world, rank=0, seed=3, peer_exchange=False)
    g = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn(stack.local, cfg.hidden, device=cuda_device, generator=g).to(torch.bfloat16)
    blk = stack.blocks[0]
    mod = stack.modulation(500.0)[0]
    hq, hs = stack._norm_quant(x, mod[0], mod[1])
    fused = stack._qkv_producer(hq, hs, blk)
    from spark_h3_b200.fp8_linear import fp8_gemm

    separate = stack._qkv_rope(fp8_gemm(hq, hs, *blk["qkv"]), blk)
    torch.cuda.synchronize()
    for a, b in zip(fused, separate):
        assert a.shape == b.shape == (world, stack.local, cfg.heads // world, 128)
        diff = (a.float() - b.float()).abs()
        assert diff.max().item() <= 2e-2 * b.float().abs().max().item() + 1e-3
        assert (a == b).float().mean().item() > 0.9  # same bf16 values but for sin/cos rounding


def _peer_worker(rank, world, port, results):
    import os
    from datetime import timedelta

    from spark_h3_b200.dit import DiTConfig, DiTStack

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        cfg = DiTConfig(hidden=256, heads=4, ffn=512, blocks=2)
        outs = []
        for peer in (True, False):
            stack = DiTStack(cfg, (2, 16, 32), device=dev, world=world, rank=rank, seed=0,
                             spark_mode="reweight_only", peer_exchange=peer)
            assert (stack.peer is not None) == peer
            g = torch.Generator(device=dev).manual_seed(100 + rank)
            x = torch.randn(stack.local, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
            for dense in (True, False, False):
                stack.step(x, 500.0, dense=dense)
            torch.cuda.synchronize()
            outs.append(x.clone())
            stack.close()
        results.put((rank, bool(torch.equal(outs[0], outs[1])), bool(torch.isfinite(outs[0]).all())))
    except Exception as e:  # pragma: no cover - reported to the parent
        results.put((rank, f"error: {e!r}", False))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_matches_nccl_two_gpus():
    """Two ranks, one per GPU: the stack with the all-to-all done by the producer's peer
    stores equals the stack with the NCCL all-to-all, bit for bit, over dense and sparse
    steps."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 29600 + (os.getpid() % 200)
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = [results.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is True and r[2] for r in got), got

"""Benchmark of one Spark-H3 sparse attention layer on B200.

Workload: B=1, grid (31, 48, 84) -> N = 124,992 tokens, H = 32, D = 128, bf16, 128-token
blocks, topk_ratio 0.1, anchor-weighted tail summaries with the log-mass correction, no
reblock.  One step = pool Q -> anchor -> pool K + summaries -> block scores + Top-K ->
sparse attention (the 64-row partial tail attends densely inside the same kernel).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload config1|config2|fp8|config4|tails|sm100_reference|summaries]

`--workload config2` times the same layer in the reference's default "full" mode at the
config-2 size (grid 61x48x84, N = 245,952, 64-token blocks, clustered content): reblock
(metric factors, features, landmark tree, head-wise permutes) + the sparse layer + the
inverse permute.  `--workload fp8` times the config-3 e4m3 linears (M = 124,992 tokens,
K = 4096, N in {12288, 4096, 16384}).  Both print one JSON line each; the default run is
config 1 only.  `--workload sm100_reference` times our attention kernel beside the
reference's own tcgen05 kernel (SparkReweightForwardSm100, installed under baseline/_ref) at
config 1 with 64-token blocks, same inputs and route, and prints both with their ratio.

With N > 1 (torchrun, one process per GPU) the 32 heads are split across ranks (strong
scaling, no data-path collective); timing is the max over ranks.  `value` is the
dense-equivalent throughput 4*N^2*H*D / time of the whole job.  Every `--gpus N` line also
carries `dit_stack`: BASELINE config 4 (the 8-block synthetic DiT at N = 245,952) run as the
19-step schedule (4 dense + 15 Spark evaluations) in one timed region, tokens split across
the ranks and heads exchanged by NCCL all-to-all, with the exchange time per sparse step.

`--impl reference` times the CPU restatement of the same layer (oracle/: the reference is
a Python/Triton project whose kernels do not run on the host) on the host cores: the route
and the summaries of all 32 heads in full, and the attention of a sample of query blocks of
one head, extrapolated to the layer.  The repo arm's `cpu_baseline` is one such step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "spark-h3_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "sparse-attn ms/layer & eff. TFLOPS @N=125k,H=32,D=128,topk0.1; DiT step s/it"
UNIT = "TFLOP/s (dense-equivalent 4*N^2*H*D per layer)"
GRID = (31, 48, 84)
HEADS = 32
PROFILE_ONLY = False
HEAD_DIM = 128
BLOCK = 128
TOPK_RATIO = 0.1
# DRAM bytes per launch of the attention kernel at this workload: dram__bytes_read.sum +
# dram__bytes_write.sum of one launch of the same layer with 4 of the 32 heads (0.662 GB read
# + 0.126 GB written), scaled by 8.  Heads run one after another through the grid, so the
# traffic grows with the head count.
ATTENTION_TRAFFIC_BYTES = 8 * (661666816 + 125626880)
# The same for the config-2 attention launch at top-k 0.1 (query blocks paired): one launch of
# the full-mode layer with 2 of the 32 heads (3.135 GB read + 0.139 GB written), scaled by 16.
CONFIG2_ATTENTION_TRAFFIC_BYTES = 16 * (3134581504 + 139380480)


def dense_flops(tokens: int, heads: int, dim: int) -> float:
    return 4.0 * tokens * tokens * heads * dim


def sparse_flops(tokens: int, heads: int, dim: int, block: int, topk: int) -> float:
    """Algorithmic FLOPs of the sparse attention kernel: every routed query row sees topk
    exact blocks plus one summary column per other key block; rows past the last complete
    block attend every key."""
    nb = math.ceil(tokens / block)
    query_tokens = (tokens // block) * block
    routed = 4.0 * query_tokens * heads * dim * (topk * block + (nb - topk))
    dense = 4.0 * (tokens - query_tokens) * tokens * heads * dim
    return routed + dense


def load_peaks() -> dict:
    """Roofline denominators.  The config-1 kernel is timed over well under a second, so
    its peak is the burst bf16 figure; the sustained one (a seconds-long loop at the power
    cap) is reported beside it."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        burst = data.get("bf16_tflops") or data.get("bf16_tflops_sustained")
        return dict(bf16=burst, bf16_sustained=data.get("bf16_tflops_sustained") or burst, hbm=data.get("hbm_gbs"),
                    source="MEASURED_PEAKS.json bf16_tflops (burst; measured, not nominal)")
    return dict(bf16=1590.0, bf16_sustained=1400.0, hbm=6650.0,
                source="fallback (1.59 PFLOP/s burst, 1.4 sustained, 6.65 TB/s)")


def config1_dict(world: int, topk: int, T: int) -> dict:
    """The config entry shared by both arms of the config-1 line."""
    nb = math.ceil(T / BLOCK)
    name = "config1" if (GRID, HEADS) == ((31, 48, 84), 32) else "config1 shape, reduced"
    return dict(workload=(f"{name}: one sparse attention layer, N={T} ({'x'.join(map(str, GRID))}), H={HEADS}, "
                          f"D={HEAD_DIM}, block {BLOCK}, topk {TOPK_RATIO} ({topk} of {T // BLOCK} blocks; {nb} with "
                          "the partial tail), reweight summaries + LSE correction, no reblock"),
                global_batch=1, seq_len=T, heads=HEADS, head_dim=HEAD_DIM, block=BLOCK, topk=topk,
                parallelism=f"heads/{world}" if world > 1 else "single GPU",
                l2="inputs (3 x 1.02 GB) exceed the 126 MB L2; no flush between steps")


DATA1 = "synthetic (seeded 8-sinusoid + 0.3 N(0,1) Q/K/V, Q scaled by 1/sqrt(D))"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict:
        mhz, max_mhz, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        mhz.sort()
        return dict(sm_mhz=mhz[len(mhz) // 2] if mhz else None, sm_max_mhz=max_mhz, reasons=sorted(reasons),
                    samples=len(mhz))


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_layer_sample(q, k, v, sample_blocks: int, summary_heads: int = 2) -> dict:
    """One config-1 layer of the CPU restatement (oracle/) on bf16 CPU tensors [1, T, H, D]:
    the route of every head in full (block means, fp32 scores, Top-K, in C with OpenMP
    threads: the restatement of the reference's own CPU route); the anchor-weighted
    summaries of `summary_heads` heads (numpy float64) and the attention of the first
    `sample_blocks` query blocks of head 0 (numpy float64), whose times are extrapolated to
    all heads and query blocks."""
    import numpy as np
    import torch

    from oracle import oracle

    host = lambda t: oracle.Tensor(t.contiguous().view(torch.int16).numpy().view(np.uint16), "bfloat16")
    oq, ok_, ov = host(q), host(k), host(v)
    _, T, H, _ = q.shape
    nb = math.ceil(T / BLOCK)
    qb = T // BLOCK
    topk = oracle.target_topk(TOPK_RATIO, qb)
    t0 = time.perf_counter()
    qc = oracle.block_means(oq, BLOCK)
    kc = oracle.key_means(ok_, BLOCK)
    a = oracle.anchor(qc, BLOCK, qb, "bfloat16")
    _, packed = oracle.topk(oracle.scores(qc, kc, qb, qb), topk, nb)
    t_route = time.perf_counter() - t0
    summary_heads = min(summary_heads, H)
    ks, vs = (host(x[:, :, :summary_heads]) for x in (k, v))
    t0 = time.perf_counter()
    ak, av, lm = oracle.summaries(np.ascontiguousarray(a[:, :summary_heads]), ks, vs, BLOCK)
    t_summ = time.perf_counter() - t0
    q0, k0, v0 = (host(x[:, :, 0:1]) for x in (q, k, v))
    t0 = time.perf_counter()
    oracle.sparse_attention(q0, k0, v0, BLOCK, np.ascontiguousarray(packed[:, :, 0:1]), ak[:, 0:1], av[:, 0:1],
                            lm[:, 0:1], qb * BLOCK, qb, qb, rows=slice(0, sample_blocks * BLOCK))
    t_attn = time.perf_counter() - t0
    factor = nb / sample_blocks * H
    summ_factor = H / summary_heads
    layer_s = t_route + t_summ * summ_factor + t_attn * factor
    return dict(value=dense_flops(T, H, HEAD_DIM) / layer_s / 1e12, unit=UNIT, cores=host_cores(), kind="port",
                layer_seconds_extrapolated=layer_s, sample_seconds=t_route + t_summ + t_attn,
                attention_extrapolation_factor=factor, summary_extrapolation_factor=summ_factor,
                sample=(f"route of all {H} heads in full ({t_route:.2f} s); summaries of {summary_heads} of {H} "
                        f"heads ({t_summ:.2f} s) x {summ_factor:.0f}; attention of {sample_blocks} of {nb} query "
                        f"blocks of one head ({t_attn:.2f} s) x {factor:.0f} ({nb}/{sample_blocks} blocks x {H} "
                        f"heads); C oracle with OpenMP and numpy/BLAS on all {host_cores()} host threads"))


def run_reference(args) -> None:
    """The reference arm: the CPU restatement of the config-1 layer on this host's cores,
    each step one cpu_layer_sample (rank 0 only; other ranks exit without work)."""
    import torch

    from spark_h3_b200.synthetic import make_qkv

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    q, k, v = make_qkv(GRID, HEADS, HEAD_DIM, seed=0, dtype=torch.bfloat16, q_scale=HEAD_DIM ** -0.5)
    samples = []
    for i in range(args.warmup + args.steps):
        base = cpu_layer_sample(q, k, v, args.cpu_sample_blocks)
        if i >= args.warmup:
            samples.append(base)
    samples.sort(key=lambda b: b["layer_seconds_extrapolated"])
    base = samples[len(samples) // 2]
    layer_s = base["layer_seconds_extrapolated"]
    T = q.shape[1]
    value = dense_flops(T, HEADS, HEAD_DIM) / layer_s / 1e12
    line = dict(metric=METRIC, value=value, unit=UNIT, impl="reference", n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=layer_s * 1e3, higher_is_better=True, scaling="strong",
                vs_baseline=None, dtype="bf16", data=DATA1,
                config=config1_dict(1, ops_target_topk(T), T),
                extrapolated=dict(layer_seconds=layer_s, sample_seconds_per_step=base["sample_seconds"],
                                  attention_extrapolation_factor=base["attention_extrapolation_factor"]),
                cpu_baseline=base, e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    emit(json.dumps(line), flush=True)


def ops_target_topk(T: int) -> int:
    qb = T // BLOCK
    return min(max(1, round(TOPK_RATIO * qb)), qb)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from spark_h3_b200 import ops
    from spark_h3_b200.sharding import max_over_ranks, shard_heads
    from spark_h3_b200.synthetic import make_qkv

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        quiet_nccl()
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if HEADS % world:
        raise SystemExit("the head count must divide evenly across GPUs")
    heads = HEADS // world

    # Inputs: generated on the device (seeded), this rank's head shard made contiguous.
    q, k, v = make_qkv(GRID, HEADS, HEAD_DIM, seed=0, device=dev, dtype=torch.bfloat16, q_scale=HEAD_DIM ** -0.5)
    q, k, v = (shard_heads(x, world, rank) for x in (q, k, v))
    torch.cuda.synchronize()
    T = q.shape[1]
    nb = math.ceil(T / BLOCK)
    qb = T // BLOCK
    topk = ops.target_topk(TOPK_RATIO, qb)
    workspace = torch.empty(ops.route_workspace_bytes(1, qb, heads, qb), device=dev, dtype=torch.uint8)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    attn_events = []

    def step(record: bool):
        qc = ops.pool_queries(q, BLOCK)
        anchor = ops.query_anchor(qc, BLOCK, qb, torch.bfloat16)
        kc, ak, av, lm = ops.pool_keys_summaries(k, v, anchor, BLOCK)
        packed, _ = ops.route_topk(qc, kc, qb, qb, topk, workspace=workspace, want_indices=False)
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ops.sparse_attention(q, k, v, BLOCK, packed, ak, av, lm, query_tokens=qb * BLOCK, sink_first=qb,
                             sink_last=qb, out=out)
        if record:
            e1.record(stream)
            attn_events.append((e0, e1))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(False)
    barrier()
    if ops.read_device_status(dev) != 0:
        raise SystemExit("a kernel wait timed out during warm-up")

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            step(True)
        stop.record(stream)
        barrier()
    elapsed_ms = start.elapsed_time(stop)
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_events) / len(attn_events)
    elapsed_ms, attn_ms = max_over_ranks([elapsed_ms, attn_ms], device=dev)
    ms_per_step = elapsed_ms / args.steps
    total_dense = dense_flops(T, HEADS, HEAD_DIM)
    value = total_dense / (ms_per_step * 1e-3) / 1e12
    if PROFILE_ONLY:
        if rank == 0:
            emit(json.dumps(dict(profile_case=True, grid=GRID, heads=HEADS, ms_per_step=ms_per_step,
                                  attention_kernel_ms=attn_ms)), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # End to end through the public API with host buffers: every step uploads Q/K/V from
    # pinned memory, runs the layer and downloads the output, streamed in head chunks so the
    # copies overlap the compute (ops.spark_layer_streamed).
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    e2e_chunks = args.e2e_chunks or next(c for c in (16, 8, 4, 2, 1) if heads % c == 0)
    if heads % e2e_chunks:
        raise SystemExit(f"--e2e-chunks {e2e_chunks} does not divide the {heads} heads of a rank")

    def e2e_step():
        ops.spark_layer_streamed(hq, hk, hv, hout, chunks=e2e_chunks, device=dev, block=BLOCK, topk_ratio=TOPK_RATIO)

    for _ in range(max(1, min(args.warmup, 2))):
        e2e_step()
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 5))
    e_start.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e_stop.record(stream)
    barrier()
    (e2e_ms,) = max_over_ranks([e_start.elapsed_time(e_stop) / e2e_steps], device=dev)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv)) * world
    d2h = hout.numel() * hout.element_size() * world

    dense_sdpa_ms = dense_clocks = None
    if world == 1 and not args.no_dense:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))
        try:
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                for _ in range(3):
                    torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
                torch.cuda.synchronize()
                d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with ClockSampler(local_rank) as sdpa_clocks:
                    d0.record(stream)
                    for _ in range(args.dense_iters):
                        torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
                    d1.record(stream)
                    torch.cuda.synchronize()
                dense_sdpa_ms = d0.elapsed_time(d1) / args.dense_iters
                dense_clocks = sdpa_clocks.summary()
        except RuntimeError as err:  # cuDNN backend unavailable
            dense_sdpa_ms = f"unavailable: {err}".splitlines()[0][:200]
        del qt, kt, vt

    status = ops.read_device_status(dev)
    cpu_inputs = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu_inputs = tuple(x.cpu() for x in (q, k, v))
    del hq, hk, hv, hout
    if rank == 0:
        peaks = load_peaks()
        flops_launch = sparse_flops(T, heads, HEAD_DIM, BLOCK, topk)
        achieved = flops_launch / (attn_ms * 1e-3) / 1e12
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=ms_per_step, higher_is_better=True, scaling="strong", vs_baseline=None, dtype="bf16",
            data=DATA1, config=config1_dict(world, topk, T),
            ms_per_layer=ms_per_step, attention_kernel_ms=attn_ms,
            sparse_flops_per_layer=sparse_flops(T, HEADS, HEAD_DIM, BLOCK, topk),
            dense_equivalent_flops_per_layer=total_dense,
            dense_cudnn_sdpa_ms=dense_sdpa_ms, dense_cudnn_sdpa_iters=args.dense_iters if dense_sdpa_ms else None,
            dense_cudnn_sdpa_clocks=dense_clocks,
            speedup_vs_dense_sdpa=(dense_sdpa_ms / ms_per_step if isinstance(dense_sdpa_ms, float) else None),
            roofline=dict(bound="tensor", kernel="sparse_attention_sm100_kernel", achieved=achieved,
                          peak=peaks["bf16"], unit="TFLOP/s", frac=achieved / peaks["bf16"],
                          frac_of_sustained=achieved / peaks["bf16_sustained"],
                          traffic=ATTENTION_TRAFFIC_BYTES if (GRID, world) == ((31, 48, 84), 1) else None,
                          traffic_unit=("bytes per launch: ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                        "4-head layer, scaled x8 to 32 heads"),
                          peak_source=peaks["source"],
                          note="achieved = algorithmic sparse FLOPs per launch / mean CUDA-event launch time"),
            e2e=dict(value=total_dense / (e2e_ms * 1e-3) / 1e12, unit=UNIT, ms_per_step=e2e_ms,
                     h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                     path=f"spark_h3_b200.ops.spark_layer_streamed on pinned host Q/K/V ({e2e_chunks} head chunks, "
                          "uploads and downloads overlapped with compute), output copied back"),
            gpu_launches=6 * args.steps,
            clocks=clocks.summary(),
            device_status=status,
        )
    del q, k, v, out, workspace
    torch.cuda.empty_cache()
    dit = None if args.no_dit else dit_schedule(args, world, rank, local_rank, dev)
    if rank == 0:
        if dit is not None:
            line["dit_stack"] = dit
        if cpu_inputs is not None:
            # one warm-up sample, then the median of three (host timings vary run to run)
            runs = [cpu_layer_sample(*cpu_inputs, args.cpu_sample_blocks) for _ in range(4)][1:]
            line["cpu_baseline"] = sorted(runs, key=lambda r: r["layer_seconds_extrapolated"])[1]
        emit(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def dit_schedule(args, world: int, rank: int, local_rank: int, dev, *, grid=None, heads: int = 32,
                 spark_mode: str = "full", peer_exchange: bool = False) -> dict:
    """BASELINE config 4 as the reference's sampling loop runs it: the 8-block synthetic DiT
    at N = 245,952 for 19 evaluations (4 dense warm-up + 15 Spark, mode "full"), timed as one
    region on every rank after one dense and two Spark warm-up evaluations; tokens are split
    across the ranks for the pointwise stages and GEMMs and heads for attention (NCCL
    all-to-all).  Returns s/it and the per-step and exchange times, each the max over ranks."""
    import torch
    import torch.distributed as dist

    from spark_h3_b200 import ops
    from spark_h3_b200.dit import DiTConfig, DiTStack
    from spark_h3_b200.sharding import max_over_ranks

    if grid is None:
        grid = tuple(int(x) for x in args.dit_grid.split(",")) if args.dit_grid else (61, 48, 84)
    cfg = DiTConfig(hidden=heads * 128, heads=heads, ffn=4 * heads * 128)
    steps, dense_steps = 19, 4
    stack = DiTStack(cfg, grid, device=dev, world=world, rank=rank, seed=0, spark_mode=spark_mode,
                     topk_ratio=TOPK_RATIO, steps=steps, peer_exchange=peer_exchange)
    exchange = ("q/k/v all-to-all by the QKV GEMM epilogue's stores to peer buffers (CUDA IPC over NVLink), output "
                "all-to-all by NCCL" if stack.peer is not None else "NCCL all-to-all (q, k, v to heads; output back "
                "to tokens)")
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(stack.local, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    stack.step(x, 999.0, dense=True)
    stack.step(x, 990.0, dense=False)
    stack.step(x, 980.0, dense=False)
    barrier()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    stack.exchange_events = [] if world > 1 else None
    with ClockSampler(local_rank) as clocks:
        barrier()
        marks[0].record(stream)
        for i in range(steps):
            stack.step(x, 1000.0 * (1.0 - i / steps), dense=i < dense_steps)
            marks[i + 1].record(stream)
        barrier()
    step_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
    total_ms = marks[0].elapsed_time(marks[steps])
    per_step = 2 * cfg.blocks  # exchanges per evaluation: to heads, back to tokens, per block
    events = stack.exchange_events or []
    a2a_ms = sum(e0.elapsed_time(e1) for e0, e1 in events[dense_steps * per_step:]) / (steps - dense_steps)
    dense_ms = sum(step_ms[:dense_steps]) / dense_steps
    sparse_ms = sum(step_ms[dense_steps:]) / (steps - dense_steps)
    total_ms, dense_ms, sparse_ms, a2a_ms = max_over_ranks([total_ms, dense_ms, sparse_ms, a2a_ms], device=dev)
    status = ops.read_device_status(dev)
    stack.close()
    del stack, x
    torch.cuda.empty_cache()
    T = grid[0] * grid[1] * grid[2]
    return dict(
        metric="DiT step s/it (config 4: 8-block synthetic DiT, 19 steps = 4 dense + 15 Spark)",
        value=total_ms / steps / 1e3, unit="s/it", higher_is_better=False, scaling="strong",
        timed="one region of all 19 evaluations (CUDA events, barrier and synchronize on both sides, max over ranks)",
        workload=(f"config4: {cfg.blocks} blocks, hidden {cfg.hidden}, {cfg.heads} heads x {cfg.head_dim}, FFN "
                  f"{cfg.ffn} GELU, e4m3 linears, N={T} ({'x'.join(map(str, grid))}), Spark mode {spark_mode}, "
                  f"topk {TOPK_RATIO}"),
        parallelism=(f"tokens/{world} for the pointwise stages and GEMMs, heads/{world} for attention, {exchange}"
                     if world > 1 else "single GPU"),
        schedule_seconds=total_ms / 1e3, dense_step_ms=dense_ms, sparse_step_ms=sparse_ms,
        all_to_all_ms_per_sparse_step=a2a_ms if world > 1 else 0.0,
        all_to_all_share_of_sparse_step=(a2a_ms / sparse_ms) if world > 1 else 0.0,
        all_to_all_bytes_per_layer=4 * T * cfg.heads * cfg.head_dim * 2 if world > 1 else 0,
        note=("exchange time = CUDA events around the four all_to_all_single calls of each block, summed over "
              "the 8 blocks; it includes waiting for the slowest rank"),
        clocks=clocks.summary(), device_status=status)


def _timed(fn, steps: int, warmup: int, stream) -> float:
    """Mean CUDA-event milliseconds of fn() over `steps` calls after `warmup` calls."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_config2(args) -> None:
    """the full Spark mode (landmark-v2 reblock + Top-K + reweight) at
    N = 245,952 on one GPU, one JSON line per top-k ratio in {0.05, 0.1, 0.2} (BASELINE's
    set; --topk-ratios to change it).  Each line carries the layer time, the attention
    kernel alone on the reblocked Q/K/V with that ratio's route, and the reblock stages."""
    import torch

    from spark_h3_b200 import ops, reblock
    from spark_h3_b200.attention import spark_attention_bthd
    from spark_h3_b200.config import H3SparseAttentionConfig
    from spark_h3_b200.layout import PackedLayout
    from spark_h3_b200.processor import _Controller
    from spark_h3_b200.synthetic import make_qkv

    if args.gpus != 1:
        raise SystemExit("--workload config2 runs on one GPU")
    grid = tuple(int(x) for x in args.grid.split(",")) if args.grid else (61, 48, 84)
    heads, block = args.heads or 32, 64
    ratios = [float(r) for r in args.topk_ratios.split(",")]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v = make_qkv(grid, heads, HEAD_DIM, seed=0, device=dev, dtype=torch.bfloat16, clustered=True)
    T = q.shape[1]
    ids = torch.arange(T)
    layout = PackedLayout(permutation=ids, inverse_permutation=ids, grid=grid, video_tokens=T, sequence_length=T,
                          video_positions=torch.zeros(T, 3, dtype=torch.long))
    stream = torch.cuda.current_stream(dev)
    layers = {}
    with ClockSampler(0) as clocks:
        for ratio in ratios:
            cfg = H3SparseAttentionConfig.spark(num_inference_steps=1000, mode="full", sol_route_topk_ratio=ratio)
            controller = _Controller(cfg)
            layers[ratio] = _timed(lambda: spark_attention_bthd(controller, q, k, v, layout, 0), args.steps,
                                   args.warmup, stream)
    clock_summary = clocks.summary()
    if args.profile_only:
        emit(json.dumps(dict(profile_case=True, workload="config2", grid=grid, heads=heads, ms_per_step=layers)),
             flush=True)
        return
    # Stage breakdown (same inputs, same stream).
    samples = torch.from_numpy(reblock.hilbert_midpoint_sample_indices(grid, T // 64).astype("int32")).to(dev)
    factors = reblock.metric_factors(q, k, samples)
    features = reblock.transform(q, k, factors, T)
    plan = reblock._plan(T, 16, grid, "power_of_two_fanout", None, None, "flat", dev)
    metric_ms = _timed(lambda: reblock.metric_factors(q, k, samples), 3, 1, stream)
    transform_ms = _timed(lambda: reblock.transform(q, k, factors, T), 3, 1, stream)
    tree_ms = _timed(lambda: plan.run(features), 3, 1, stream)
    reblock.transform(q, k, factors, T, out=plan.features_buffer(2 * heads))
    tree_graph_ms = _timed(lambda: plan.replay(2 * heads), 3, 1, stream)  # captured CUDA graph
    del features
    qp, qi, kp, ki, _ = reblock.qk_block_permutations(q, k, T, grid)
    permute_ms = _timed(lambda: [ops.headwise_permute(t, p, T) for t, p in ((q, qp), (k, kp), (v, kp))], 3, 1,
                        stream)
    q2, k2, v2 = (ops.headwise_permute(t, p, T) for t, p in ((q, qp), (k, kp), (v, kp)))
    del q, k, v
    qc = ops.pool_queries(q2, block)
    anchor = ops.query_anchor(qc, block, T // block, torch.bfloat16)
    _, ak, av, lm = ops.pool_keys_summaries(k2, v2, anchor, block)
    kc = ops.pool_keys_summaries(k2, None, None, block, want_summaries=False)[0]
    out = torch.empty_like(q2)
    peaks = load_peaks()
    rows = 2 * heads
    transform_bytes = rows * T * HEAD_DIM * 2 * 2  # read Q or K rows, write the features
    nb = T // block
    stages = dict(reblock_metric=metric_ms, reblock_transform=transform_ms, reblock_tree=tree_ms,
                  reblock_tree_graph=tree_graph_ms, qkv_permutes=permute_ms)
    transform_roofline = dict(
        bound="hbm", kernel="reblock_transform_kernel", achieved=transform_bytes / (transform_ms * 1e-3) / 1e9,
        peak=peaks["hbm"], unit="GB/s", frac=transform_bytes / (transform_ms * 1e-3) / 1e9 / peaks["hbm"],
        traffic=None, peak_source="MEASURED_PEAKS.json hbm_gbs (copy bandwidth, measured)",
        note="algorithmic bytes: 64 rows x N x 128 x 2 B read + the same written")
    for ratio in ratios:
        topk = ops.target_topk(ratio, nb)
        packed, _ = ops.route_topk(qc, kc, nb, nb, topk, want_indices=False)
        pairs = ops.route_pairs(packed, nb)  # the layer pairs the query blocks; the kernel alone is timed below
        attn = lambda: ops.sparse_attention(q2, k2, v2, block, packed, ak, av, lm, query_tokens=nb * block,
                                            sink_first=nb, sink_last=nb, out=out, pairs=pairs)
        with ClockSampler(0) as attn_clocks:
            attn_ms = _timed(attn, args.steps, args.warmup, stream)
        flops = sparse_flops(T, heads, HEAD_DIM, block, topk)
        achieved = flops / (attn_ms * 1e-3) / 1e12
        ms = layers[ratio]
        line = dict(
            metric=METRIC + " [config 2: full mode with reblock]",
            value=dense_flops(T, heads, HEAD_DIM) / (ms * 1e-3) / 1e12, unit=UNIT, n_gpus=1, steps=args.steps,
            warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="strong", vs_baseline=None,
            dtype="bf16",
            data="synthetic (seeded 8-sinusoid + clustered content: 64 N(0,1) centroids on a 4x4x4 region "
                 "partition, 0.25 N(0,1) noise)",
            config=dict(workload=f"config2: mode full (landmark-v2 reblock, Top-K {ratio}, reweight), N={T} "
                                 f"({'x'.join(map(str, grid))}), H={heads}, D=128, block 64",
                        seq_len=T, heads=heads, block=block, topk_ratio=ratio, topk=topk,
                        l2="inputs (3 x 2.0 GB) exceed the 126 MB L2; no flush between steps"),
            ms_per_layer=ms, attention_kernel_ms=attn_ms, sparse_flops_per_layer=flops,
            dense_equivalent_flops_per_layer=dense_flops(T, heads, HEAD_DIM),
            stages_ms=stages,
            roofline=dict(bound="tensor", kernel="sparse_attention_sm100_kernel", achieved=achieved,
                          peak=peaks["bf16"], unit="TFLOP/s", frac=achieved / peaks["bf16"],
                          frac_of_sustained=achieved / peaks["bf16_sustained"],
                          traffic=(CONFIG2_ATTENTION_TRAFFIC_BYTES
                                   if (grid, heads, ratio) == ((61, 48, 84), 32, 0.1) else None),
                          traffic_unit=("bytes per launch: ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                        "2-head layer at top-k 0.1, scaled x16 to 32 heads"),
                          peak_source=peaks["source"],
                          note="sparse FLOPs 4 D (k 64 + (n - k)) per routed query row; the kernel's 128-row tiles "
                               "pair two 64-row query blocks and compute the union of their key sets"),
            reblock_transform_roofline=transform_roofline,
            clocks=clock_summary, attention_clocks=attn_clocks.summary(),
            device_status=ops.read_device_status(dev))
        emit(json.dumps(line), flush=True)


def run_tails(args) -> None:
    """The Spark layer at config-1 size (N = 124,992, H = 32, D = 128, bf16) with the
    reference's 64-token blocks, per tail granularity (query / block / block8x8) and summary
    numerics: CUDA-event ms per layer, inputs resident in HBM."""
    import torch

    from spark_h3_b200 import ops
    from spark_h3_b200.synthetic import make_qkv

    if args.gpus != 1:
        raise SystemExit("--workload tails runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    grid = tuple(int(x) for x in args.grid.split(",")) if args.grid else GRID
    heads = args.heads or HEADS
    q, k, v = make_qkv(grid, heads, HEAD_DIM, seed=0, device=dev, dtype=torch.bfloat16, q_scale=HEAD_DIM ** -0.5)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    cases = [("query", "tensorcore", "stored"), ("query", "comfy_fp32", "pre_round"), ("block", "tensorcore", "stored"),
             ("block8x8", "tensorcore", "stored")]
    ms = {}
    with ClockSampler(0) as clocks:
        for tail, math_, key in cases:
            layer = lambda: ops.spark_layer(q, k, v, block=64, topk_ratio=TOPK_RATIO, out=out, tail_granularity=tail,
                                            summary_math=math_, logmass_key=key)
            ms[f"{tail}/{math_}/{key}"] = _timed(layer, args.steps, args.warmup, stream)
    status = ops.read_device_status(dev)
    T = q.shape[1]
    emit(json.dumps(dict(
        metric="Spark layer ms per tail granularity and summary numerics (ablations)", value=ms["block/tensorcore/stored"],
        unit="ms", n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms["block/tensorcore/stored"],
        higher_is_better=False, scaling="strong", vs_baseline=None, dtype="bf16",
        data="synthetic (seeded 8-sinusoid + 0.3 N(0,1) Q/K/V)",
        config=dict(workload=f"tails: N={T} ({'x'.join(map(str, grid))}), H={heads}, D=128, block 64, topk {TOPK_RATIO}"),
        ms_per_layer=ms, clocks=clocks.summary(), device_status=status)), flush=True)


def run_fp8(args) -> None:
    """e4m3 linears with per-token x per-output-channel scales."""
    import torch

    from spark_h3_b200 import ops
    from spark_h3_b200.fp8_linear import fp8_gemm, quantize_rows, quantize_weight

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    M, K = args.fp8_rows, 4096
    g = torch.Generator(device=dev).manual_seed(0)
    x = (torch.randn(M, K, device=dev, generator=g)
         * torch.empty(M, 1, device=dev).log_normal_(0.0, 0.5, generator=g)).to(torch.bfloat16)
    peaks = load_peaks()
    fp8_peak = 2 * peaks["bf16"]
    shapes = {}
    with ClockSampler(0) as clocks:
        quant_ms = _timed(lambda: quantize_rows(x), args.steps, args.warmup, stream)
        xq, xs = quantize_rows(x)
        for N in (12288, 4096, 16384):
            w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            wq, ws = quantize_weight(w)
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            gemm_ms = _timed(lambda: fp8_gemm(xq, xs, wq, ws, out=out), args.steps, args.warmup, stream)
            flops = 2.0 * M * N * K
            entry = dict(gemm_ms=gemm_ms, tflops=flops / (gemm_ms * 1e-3) / 1e12)
            try:
                one = torch.ones(1, 1, device=dev)
                lib_ms = _timed(lambda: torch._scaled_mm(xq, wq.t(), scale_a=one, scale_b=one,
                                                         out_dtype=torch.bfloat16, use_fast_accum=True),
                                args.steps, args.warmup, stream)
                entry["cublas_scaled_mm_per_tensor_ms"] = lib_ms
                row_ms = _timed(lambda: torch._scaled_mm(xq, wq.t(), scale_a=xs, scale_b=ws.reshape(1, -1),
                                                         out_dtype=torch.bfloat16, use_fast_accum=True),
                                args.steps, args.warmup, stream)
                entry["torch_scaled_mm_rowwise_ms"] = row_ms
            except RuntimeError as err:
                entry["library"] = f"unavailable: {err}".splitlines()[0][:160]
            entry["bf16_matmul_ms"] = _timed(lambda: x @ w.t(), 2, 1, stream)
            shapes[f"{K}->{N}"] = entry
            del w, wq, out
    total_flops = sum(2.0 * M * int(key.split("->")[1]) * K for key in shapes)
    total_ms = sum(e["gemm_ms"] for e in shapes.values()) + 3 * quant_ms
    best = max(shapes.values(), key=lambda e: e["tflops"])
    status = ops.read_device_status(dev)
    line = dict(
        metric="fp8_linear e4m3 TFLOP/s (config 3: M=124992, K=4096, N in {12288, 4096, 16384})",
        value=total_flops / (total_ms * 1e-3) / 1e12, unit="TFLOP/s (2*M*N*K, quantisation included)",
        n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=total_ms, higher_is_better=True,
        scaling="strong", vs_baseline=None, dtype="e4m3 inputs, fp32 accumulate, bf16 out",
        data="synthetic: X ~ N(0,1) x LogNormal(0,0.5) per token, W ~ N(0,0.02)",
        config=dict(workload="config3: three e4m3 linears per step with one per-token quantisation each", M=M, K=K),
        quantize_rows_ms=quant_ms,
        quantize_rows_gbs=(M * K * 3) / (quant_ms * 1e-3) / 1e9,
        shapes=shapes,
        roofline=dict(bound="tensor", kernel="fp8_gemm_kernel", achieved=best["tflops"], peak=fp8_peak,
                      unit="TFLOP/s", frac=best["tflops"] / fp8_peak, traffic=None,
                      peak_source="2 x " + peaks["source"] + " (e4m3 issues at twice the bf16 rate)"),
        clocks=clocks.summary(), device_status=status)
    emit(json.dumps(line), flush=True)


_JSON_OUT = None


def run_summaries(args) -> None:
    """The bf16 key/value summaries kernel alone (key means, anchor logits, AK / AV / LM),
    CUDA-event ms per call and HBM GB/s for K and V read once, at config 1 (128- and 64-token
    blocks) and config 2 (64-token blocks); a SHA-256 prefix of the outputs for bit-for-bit
    comparisons between builds."""
    import hashlib

    import torch

    from spark_h3_b200 import ops
    from spark_h3_b200.synthetic import make_qkv

    if args.gpus != 1:
        raise SystemExit("--workload summaries runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak = load_peaks()["hbm"]
    cases = {}
    for name, block, grid in (("config1_block128", 128, (31, 48, 84)), ("config1_block64", 64, (31, 48, 84)),
                              ("config2_block64", 64, (61, 48, 84))):
        q, k, v = make_qkv(grid, HEADS, HEAD_DIM, seed=0, device=dev, dtype=torch.bfloat16, q_scale=HEAD_DIM ** -0.5)
        n = q.shape[1] // block
        anchor = ops.query_anchor(ops.pool_queries(q, block), block, n, q.dtype)
        del q
        call = lambda: ops.pool_keys_summaries(k, v, anchor, block)
        digest = hashlib.sha256()
        for t in call():
            digest.update(t.contiguous().view(torch.uint8).cpu().numpy().tobytes())
        ms = _timed(call, args.steps, args.warmup, stream)
        gbs = 2 * k.numel() * k.element_size() / ms / 1e6
        cases[name] = dict(ms=ms, gbs=gbs, frac_of_measured_copy=gbs / peak, sha256_16=digest.hexdigest()[:16])
        del k, v, anchor
    emit(json.dumps(dict(
        metric="kv summaries kernel ms per call (K and V read once)", value=cases["config1_block128"]["ms"], unit="ms",
        n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=cases["config1_block128"]["ms"],
        higher_is_better=False, scaling="strong", vs_baseline=None, dtype="bf16", data=DATA1,
        config=dict(workload="kv summaries: H=32, D=128; config 1 (N=124992) and config 2 (N=245952)",
                    l2="K and V (2.05 / 4.03 GB) exceed the 126 MB L2; no flush between calls"),
        cases=cases, device_status=ops.read_device_status(dev))), flush=True)


def _import_reference_sm100():
    """The reference's fused SM100 attention (`SparkReweightForwardSm100`, reached through
    `h3_sparse_attention/sol_numerator_virtual_q.py::virtual_q_attention` with
    H3_SPARK_REWEIGHT_FUSED=1) from the installed copy under baseline/_ref.  The reference's
    code is not changed.  One adapter sits in front of it: the CuTe DSL in this image returns
    a compiled callable whose parameters are positional only, while the reference passes
    `stream=` by keyword, so the adapter hands the stream over positionally."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "h3_sparse_attention").is_dir():
        raise SystemExit("--workload sm100_reference needs the reference installed under baseline/_ref")
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    os.environ["H3_SPARK_REWEIGHT_FUSED"] = "1"
    import cutlass.cute as cute

    compile_ = cute.compile

    class _StreamPositional:
        def __init__(self, fn):
            self.fn = fn

        def __call__(self, *a, stream=None):
            return self.fn(*a) if stream is None else self.fn(*a, stream)

    cute.compile = lambda *a, **kw: _StreamPositional(compile_(*a, **kw))
    import h3_sparse_attention.sol_numerator_virtual_q as rw
    from sol_attn.preprocess import _reduce_kv

    return rw, _reduce_kv


def run_sm100_reference(args) -> None:
    """Config 1 at the reference's 64-token blocks: our attention kernel beside the
    reference's own tcgen05/TMEM kernel, on the same Q/K/V and the same route, on one GPU.

    One parent range covers the sequence; our route (pool, anchor, summaries, Top-K) is
    unpacked into the reference's dense uint8 route, and the reference receives its own
    anchors and summaries (`build_virtual_anchors`, `virtual_summaries`) precomputed, so both
    timed calls are the attention kernel alone.  The reference is also timed with its
    summaries inside the call.  Outputs are compared (max abs, cosine) before timing.  Each
    launch is timed alone with CUDA events after a device sleep, median of `--steps`."""
    import torch

    from spark_h3_b200 import ops
    from spark_h3_b200.synthetic import make_qkv

    if args.gpus != 1:
        raise SystemExit("--workload sm100_reference runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rw, reduce_kv = _import_reference_sm100()
    grid = tuple(int(x) for x in args.grid.split(",")) if args.grid else GRID
    heads = args.heads or HEADS
    block = 64
    q, k, v = make_qkv(grid, heads, HEAD_DIM, seed=0, device=dev, dtype=torch.bfloat16, q_scale=HEAD_DIM ** -0.5)
    B, T, H, D = q.shape
    n = T // block
    qc = ops.pool_queries(q, block)
    anchor = ops.query_anchor(qc, block, n, q.dtype)
    kc, ak, av, lm = ops.pool_keys_summaries(k, v, anchor, block)
    topk = ops.target_topk(TOPK_RATIO, n)
    packed, _ = ops.route_topk(qc, kc, n, n, topk)
    pairs = ops.route_pairs(packed, n)
    out = torch.empty_like(q)

    def ours():
        return ops.sparse_attention(q, k, v, block, packed, ak, av, lm, query_tokens=T, sink_first=n, sink_last=n,
                                    out=out, pairs=pairs)[0]

    ranges = torch.tensor([[0, T]], device=dev, dtype=torch.int64)
    mapping = torch.zeros(n, device=dev, dtype=torch.int64)
    dense_route = rw.unpack_packed_route(packed, n)
    kc_ref, _ = reduce_kv(k, v)
    anchors_ref = rw.build_virtual_anchors(q, ranges)
    summaries_ref = rw.virtual_summaries(anchors_ref, k, v)

    def ref(precomputed: bool):
        kw = dict(virtual_anchors=anchors_ref, precomputed_summaries=summaries_ref) if precomputed else {}
        return rw.virtual_q_attention(q, k, v, virtual_ranges=ranges, leaf_to_virtual=mapping, key_centroids=kc_ref,
                                      route=dense_route, sink_tokens=0, force_local_blocks=False, **kw)

    t0 = time.time()
    o_ref = ref(True)
    torch.cuda.synchronize()
    compile_s = time.time() - t0
    o_ours = ours()
    torch.cuda.synchronize()
    diff = (o_ours.float() - o_ref.float()).abs()
    a, b = o_ours.float().flatten(), o_ref.float().flatten()
    cosine = float((a @ b) / (a.norm() * b.norm() + 1e-30))
    max_abs, mean_abs = float(diff.max()), float(diff.mean())
    del diff, a, b

    def each(fn, iters):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ts = []
        for _ in range(iters):
            torch.cuda._sleep(2_000_000)  # the host's enqueue stays outside the timed interval
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2], ts

    with ClockSampler(0) as clocks:
        ours_ms, ours_raw = each(ours, args.steps)
        ref_ms, ref_raw = each(lambda: ref(True), args.steps)
        ref_full_ms, _ = each(lambda: ref(False), max(3, args.steps // 2))
    status = ops.read_device_status(dev)
    flops = sparse_flops(T, H, D, block, topk)
    emit(json.dumps(dict(
        metric="attention kernel ms at config 1 with 64-token blocks: ours beside the reference's SM100 kernel",
        value=ours_ms, unit="ms", n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ours_ms,
        higher_is_better=False, scaling="strong", vs_baseline=None, dtype="bf16",
        data="synthetic (seeded 8-sinusoid + 0.3 N(0,1) Q/K/V, Q scaled by 1/sqrt(D))",
        config=dict(workload=f"config1 at block 64: N={T} ({'x'.join(map(str, grid))}), H={H}, D={D}, topk {topk} "
                             f"of {n} blocks, one parent range, no sinks", block=block, topk=topk,
                    l2="inputs (3 x 1.02 GB at full size) exceed the 126 MB L2; no flush between launches"),
        reference=dict(kernel="SparkReweightForwardSm100 via virtual_q_attention (H3_SPARK_REWEIGHT_FUSED=1)",
                       attention_ms=ref_ms, with_summaries_ms=ref_full_ms, first_call_s=round(compile_s, 1)),
        ref_ms_over_ours_ms=ref_ms / ours_ms,
        tflops=dict(ours=flops / ours_ms * 1e-9, reference=flops / ref_ms * 1e-9,
                    note="algorithmic sparse FLOPs of our exact-block + summary work at this route"),
        parity=dict(max_abs=max_abs, mean_abs=mean_abs, cosine=cosine),
        raw_ms=dict(ours=ours_raw, reference=ref_raw), clocks=clocks.summary(), device_status=status)), flush=True)


def keep_stdout_for_json() -> None:
    """The JSON line is the only thing this program writes to its stdout: the real stdout is
    kept on a private descriptor and fd 1 is pointed at stderr, so banners that libraries
    print to fd 1 (NCCL's version line among them) cannot mix into it."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w", buffering=1)
        os.dup2(2, 1)


def emit(text: str, flush: bool = True) -> None:
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(text + "\n")
    if flush:
        out.flush()


def quiet_nccl() -> None:
    """Keep stdout to the one JSON line: NCCL's version banner and warnings go to stderr."""
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")


def run_config4(args) -> None:
    """BASELINE config 4 on its own: the 19-step DiT schedule of dit_schedule, one JSON line
    with s/it as the value (torchrun for N > 1)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        quiet_nccl()
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    grid = tuple(int(x) for x in args.grid.split(",")) if args.grid else (61, 48, 84)
    dit = dit_schedule(args, world, rank, local_rank, dev, grid=grid, heads=args.heads or 32,
                       spark_mode=args.spark_mode, peer_exchange=args.peer_exchange)
    if rank == 0:
        line = dict(metric=dit.pop("metric"), value=dit.pop("value"), unit=dit.pop("unit"), n_gpus=world,
                    steps=19, warmup=3, ms_per_step=dit["schedule_seconds"] * 1e3 / 19,
                    higher_is_better=dit.pop("higher_is_better"), scaling=dit.pop("scaling"), vs_baseline=None,
                    dtype="e4m3 linears, bf16 activations and attention",
                    data="synthetic: latent tokens N(0,1), weights N(0,0.02), seeded",
                    config=dict(workload=dit.pop("workload"), parallelism=dit.pop("parallelism")), **dit)
        emit(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main():
    keep_stdout_for_json()
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-dense", action="store_true", help="skip the dense cuDNN SDPA comparison")
    ap.add_argument("--dense-iters", type=int, default=10, help="timed iterations of the dense cuDNN SDPA")
    ap.add_argument("--no-dit", action="store_true", help="skip the config-4 DiT schedule (dit_stack)")
    ap.add_argument("--dit-grid", type=str, default=None,
                    help="T,H,W token grid of the dit_stack schedule (default 61,48,84)")
    ap.add_argument("--e2e-chunks", type=int, default=0,
                    help="head chunks of the end-to-end streamed layer (0: 16 or the largest that divides)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle baseline")
    ap.add_argument("--cpu-sample-blocks", type=int, default=16,
                    help="query blocks of the one-head CPU attention sample (cpu_baseline and --impl reference)")
    ap.add_argument("--grid", type=str, default=None,
                    help="T,H,W token grid for a smaller profiling case (default 31,48,84)")
    ap.add_argument("--heads", type=int, default=None, help="head count for a smaller profiling case")
    ap.add_argument("--profile-only", action="store_true",
                    help="run only the device-resident steps (for ncu captures of a small case)")
    ap.add_argument("--workload", choices=("config1", "config2", "fp8", "config4", "tails", "sm100_reference",
                                           "summaries"),
                    default="config1",
                    help="config1 (default, the headline layer), config2 (full mode with reblock), fp8 (config 3), "
                         "config4 (DiT block stack, multi-GPU with torchrun), tails (tail granularity ablations), "
                         "sm100_reference (our attention beside the reference's SM100 kernel, block 64), "
                         "summaries (the K/V summaries kernel alone)")
    ap.add_argument("--spark-mode", default="full", help="Spark mode of the config-4 sparse steps")
    ap.add_argument("--peer-exchange", action="store_true",
                    help="config 4: the QKV producer's epilogue stores q/k/v to the owners' buffers over NVLink "
                         "instead of the NCCL all-to-all")
    ap.add_argument("--fp8-rows", type=int, default=124992, help="token rows M of the fp8 workload")
    ap.add_argument("--topk-ratios", type=str, default="0.05,0.1,0.2",
                    help="config 2: the top-k ratios, one JSON line each")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # at least three untimed warm-up steps
    global GRID, HEADS, PROFILE_ONLY
    if args.grid:
        GRID = tuple(int(x) for x in args.grid.split(","))
    if args.heads:
        HEADS = args.heads
    PROFILE_ONLY = args.profile_only
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config2":
        run_config2(args)
    elif args.workload == "fp8":
        run_fp8(args)
    elif args.workload == "config4":
        run_config4(args)
    elif args.workload == "tails":
        run_tails(args)
    elif args.workload == "sm100_reference":
        run_sm100_reference(args)
    elif args.workload == "summaries":
        run_summaries(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Synthetic DiT block stack on B200, token-sharded across the GPUs of
one node with a sequence-to-head all-to-all around attention (Ulysses style).

The reference has no such model on its attention path (its DiT is diffusers' MiniMax-H3); the
stack here is the minimal block BASELINE names: hidden 4096, 32 heads of 128, GELU FFN 16384,
RMSNorm, 3-D RoPE over (t, h, w), adaLN timestep modulation, e4m3 linears (per-token x
per-channel scales), random-init weights N(0, 0.02).  Per block and rank (Nloc = N / P
tokens, P ranks):

    x  ->  norm + modulate + quantise  ->  fused QKV GEMM  ->  q/k RMSNorm + RoPE
       ->  all-to-all (tokens -> heads)  ->  attention on all N tokens, H / P heads
       ->  all-to-all (heads -> tokens)  ->  out GEMM, x += gate1 * (.)
       ->  norm + modulate + quantise  ->  up GEMM  ->  GELU + quantise
       ->  down GEMM, x += gate2 * (.)

Attention is dense (cuDNN SDPA, as the reference's dense warmup evaluations) or the Spark
layer (spark_attention_bthd).  Every other stage runs in libsparkh3b200.so.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib
from .fp8_linear import FP8_DTYPE, fp8_gemm, quantize_weight
from .ops import _stream


@dataclass(frozen=True)
class DiTConfig:
    hidden: int = 4096
    heads: int = 32
    head_dim: int = 128
    ffn: int = 16384
    blocks: int = 8
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_bands: tuple = (32, 48, 48)  # head-dimension slices rotated by t, h, w
    t_dim: int = 256


def rope_tables(cfg: DiTConfig, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(inv_freq [D/2] fp32, axis [D/2] int8): pair j of the head dimension rotates by
    coord[axis[j]] * inv_freq[j]; each band of the head dimension uses its own frequencies."""
    if sum(cfg.rope_bands) != cfg.head_dim or any(b % 2 for b in cfg.rope_bands):
        raise ValueError("rope bands must be even and cover the head dimension")
    inv, axis = [], []
    for a, band in enumerate(cfg.rope_bands):
        for i in range(band // 2):
            inv.append(cfg.rope_theta ** (-(2.0 * i) / band))
            axis.append(a)
    return (torch.tensor(inv, dtype=torch.float32, device=device),
            torch.tensor(axis, dtype=torch.int8, device=device))


def token_coords(grid, start: int, count: int, device) -> torch.Tensor:
    """(t, h, w) of raster tokens [start, start + count) of a THW grid, int32 [count, 3]."""
    _, H_, W_ = grid
    ids = torch.arange(start, start + count, device=device, dtype=torch.int64)
    return torch.stack((ids // (H_ * W_), (ids // W_) % H_, ids % W_), dim=-1).to(torch.int32).contiguous()


def timestep_embedding(t: float, dim: int, device) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=device, dtype=torch.float32) / half)
    args = t * freqs
    return torch.cat([torch.cos(args), torch.sin(args)])


# ---------------------------------------------------------------- sequence <-> head exchange
def exchange_to_heads(send: torch.Tensor, group=None) -> torch.Tensor:
    """send [P, Nloc, Hp, D] (block p = this rank's tokens for rank p's heads) -> [P * Nloc,
    Hp, D]: every token, in order, for this rank's heads."""
    P = send.shape[0]
    if P == 1:
        return send.reshape(-1, *send.shape[2:])
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.reshape(-1, *send.shape[2:])


def exchange_to_tokens(out: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """out [N, Hp, D] (this rank's heads, every token) -> [P, Nloc, Hp, D]: block p = this
    rank's tokens for rank p's heads (the segment layout sb_fp8_quantize_segments reads)."""
    send = out.reshape(world, -1, *out.shape[1:]).contiguous()
    if world == 1:
        return send
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv


class _DeviceBuffer:
    """A torch view of a raw device allocation (bf16 as uint16 through the CUDA array
    interface, then viewed back)."""

    def __init__(self, ptr: int, shape, device):
        self.__cuda_array_interface__ = dict(shape=tuple(shape), typestr="<u2", data=(ptr, False), version=3,
                                             strides=None)
        self.device = device

    def tensor(self) -> torch.Tensor:
        return torch.as_tensor(self, device=self.device).view(torch.bfloat16)


class PeerExchange:
    """Receive buffers for q, k and v [P, Nloc, Hp, D] that every rank's QKV producer writes
    into directly over NVLink (the all-to-all done by the GEMM epilogue): allocated here,
    mapped into the other processes of the node with CUDA IPC, and listed in a device table
    [3][P] for the kernel."""

    def __init__(self, shape, device, world: int, rank: int, group=None):
        import ctypes

        self.shape, self.device, self.world, self.rank = tuple(shape), torch.device(device), world, rank
        nbytes = int(math.prod(self.shape)) * 2
        self.local, self.opened = [], []
        handles = []
        for _ in range(3):
            ptr = ctypes.c_void_p()
            _lib.call("sb_ipc_alloc", nbytes, ctypes.byref(ptr))
            self.local.append(ptr.value)
            h = (ctypes.c_uint8 * 64)()
            _lib.call("sb_ipc_handle", ptr.value, h)
            handles.append(bytes(h))
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        table = []
        for sec in range(3):
            for r in range(world):
                if r == rank:
                    table.append(self.local[sec])
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(gathered[r][sec])
                ptr = ctypes.c_void_p()
                _lib.call("sb_ipc_open", h, ctypes.byref(ptr))
                table.append(ptr.value)
                self.opened.append(ptr.value)
        self.table = torch.tensor(table, dtype=torch.int64, device=self.device)
        self.views = [_DeviceBuffer(ptr, self.shape, self.device).tensor() for ptr in self.local]
        self.flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.group = group

    def barrier(self):
        """Stream-ordered: returns once every rank's producer kernel before it has completed."""
        dist.all_reduce(self.flag, group=self.group)

    def close(self):
        """Unmap the peers' buffers, wait for every rank to do the same, free ours."""
        torch.cuda.synchronize(self.device)
        for ptr in self.opened:
            _lib.call("sb_ipc_close", ptr)
        self.opened = []
        dist.barrier(group=self.group)
        self.views = []
        for ptr in self.local:
            _lib.call("sb_ipc_free", ptr)
        self.local = []


class DiTStack:
    """The block stack on one rank.  Weights are generated from `seed` identically on every
    rank (so a P-rank run computes the same model as a 1-rank run) and kept only as e4m3
    codes with per-channel scales."""

    def __init__(self, cfg: DiTConfig, grid, *, device, world: int = 1, rank: int = 0, group=None, seed: int = 0,
                 spark_mode: str = "full", topk_ratio: float = 0.1, steps: int = 19, fused_producer: bool = True,
                 peer_exchange: bool = False):
        from .config import H3SparseAttentionConfig
        from .layout import PackedLayout
        from .processor import _Controller

        self.cfg, self.grid, self.device = cfg, tuple(grid), torch.device(device)
        self.world, self.rank, self.group = world, rank, group
        self.tokens = grid[0] * grid[1] * grid[2]
        if self.tokens % world or cfg.heads % world:
            raise ValueError("tokens and heads must split evenly across ranks")
        self.local = self.tokens // world
        self.hp = cfg.heads // world
        g = torch.Generator(device=self.device).manual_seed(seed)
        C, HD = cfg.hidden, cfg.heads * cfg.head_dim

        def linear(out_f, in_f):
            w = (torch.randn(out_f, in_f, device=self.device, generator=g) * 0.02).to(torch.bfloat16)
            return quantize_weight(w)

        self.blocks = []
        for _ in range(cfg.blocks):
            self.blocks.append(dict(
                qkv=linear(3 * HD, C), out=linear(C, HD), up=linear(cfg.ffn, C), down=linear(C, cfg.ffn),
                norm_q=(1 + 0.02 * torch.randn(cfg.head_dim, device=self.device, generator=g)).contiguous(),
                norm_k=(1 + 0.02 * torch.randn(cfg.head_dim, device=self.device, generator=g)).contiguous(),
                ada=(torch.randn(6 * C, cfg.t_dim, device=self.device, generator=g) * 0.02).contiguous()))
        self.inv_freq, self.axis = rope_tables(cfg, self.device)
        self.coords = token_coords(self.grid, rank * self.local, self.local, self.device)
        # (cos, sin) of every pair and coordinate value, for the GEMM-epilogue producer
        self.fused_producer = fused_producer and cfg.heads % 2 == 0
        self.rope_stride = max(self.grid)
        ang = torch.arange(self.rope_stride, device=self.device, dtype=torch.float32)[None, :] * self.inv_freq[:, None]
        self.rope = torch.stack((torch.cos(ang), torch.sin(ang)), dim=-1).contiguous()  # [D/2, stride, 2]
        sparse_cfg = H3SparseAttentionConfig.spark(num_inference_steps=steps, mode=spark_mode,
                                                   sol_route_topk_ratio=topk_ratio)
        self.controller = _Controller(sparse_cfg)
        # With several ranks and peer_exchange, the producer's epilogue stores q, k, v into the
        # owners' receive buffers itself; by default NCCL's all-to-all moves them (measured
        # slightly faster at 2 GPUs: its large transfers beat the epilogue's 16-byte row stores).
        self.peer = None
        if world > 1 and peer_exchange and self.fused_producer:
            self.peer = PeerExchange((world, self.local, self.hp, cfg.head_dim), self.device, world, rank, group)
        # When a list, every sequence<->head exchange appends its (start, end) CUDA events.
        self.exchange_events = None
        ids = torch.arange(self.tokens)
        self.layout = PackedLayout(permutation=ids, inverse_permutation=ids, grid=self.grid, video_tokens=self.tokens,
                                   sequence_length=self.tokens, video_positions=torch.zeros(self.tokens, 3,
                                                                                             dtype=torch.long))

    # -------------------------------------------------------------- kernels of one block
    def _norm_quant(self, x, shift, scale):
        M, C = x.shape
        q = torch.empty((M, C), device=self.device, dtype=FP8_DTYPE)
        s = torch.empty((M, 1), device=self.device, dtype=torch.float32)
        _lib.call("sb_dit_norm_modulate_quantize", x.data_ptr(), shift.data_ptr(), scale.data_ptr(), M, C,
                  float(self.cfg.eps), q.data_ptr(), s.data_ptr(), _stream(self.device))
        return q, s

    def _gemm_residual(self, a, a_scale, w, x, gate):
        codes, scale = w
        M, K = a.shape
        _lib.call("sb_fp8_gemm_residual", a.data_ptr(), a_scale.data_ptr(), 1, codes.data_ptr(), scale.data_ptr(), 1,
                  M, codes.shape[0], K, None, x.data_ptr(), gate.data_ptr(), x.data_ptr(), 0, _stream(self.device))
        return x

    def _qkv_rope(self, qkv, blk):
        cfg = self.cfg
        shape = (self.world, self.local, self.hp, cfg.head_dim)
        q, k, v = (torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in range(3))
        _lib.call("sb_dit_qkv_norm_rope", qkv.data_ptr(), blk["norm_q"].data_ptr(), blk["norm_k"].data_ptr(),
                  self.coords.data_ptr(), self.inv_freq.data_ptr(), self.axis.data_ptr(), self.local, cfg.heads,
                  cfg.head_dim, self.world, float(cfg.eps), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                  _stream(self.device))
        return q, k, v

    def _qkv_producer(self, hq, hs, blk):
        """The QKV projection with q/k RMSNorm and RoPE in its epilogue, written straight into
        the all-to-all send layout (sb_fp8_gemm_qkv_rope)."""
        cfg = self.cfg
        codes, scale = blk["qkv"]
        shape = (self.world, self.local, self.hp, cfg.head_dim)
        q, k, v = (torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in range(3))
        _lib.call("sb_fp8_gemm_qkv_rope", hq.data_ptr(), hs.data_ptr(), codes.data_ptr(), scale.data_ptr(), self.local,
                  cfg.heads, hq.shape[1], None, blk["norm_q"].data_ptr(), blk["norm_k"].data_ptr(), self.rope.data_ptr(),
                  self.rope_stride, self.coords.data_ptr(), self.axis.data_ptr(), self.world, float(cfg.eps),
                  q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, _stream(self.device))
        return q, k, v

    def _qkv_producer_peers(self, hq, hs, blk):
        """The producer with the all-to-all in its epilogue: every head row goes straight to
        its owner's receive buffer (sb_fp8_gemm_qkv_rope_peers)."""
        cfg = self.cfg
        codes, scale = blk["qkv"]
        _lib.call("sb_fp8_gemm_qkv_rope_peers", hq.data_ptr(), hs.data_ptr(), codes.data_ptr(), scale.data_ptr(),
                  self.local, cfg.heads, hq.shape[1], None, blk["norm_q"].data_ptr(), blk["norm_k"].data_ptr(),
                  self.rope.data_ptr(), self.rope_stride, self.coords.data_ptr(), self.axis.data_ptr(), self.world,
                  self.rank, float(cfg.eps), self.peer.table.data_ptr(), 0, _stream(self.device))

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _attention(self, q, k, v, layer: int, dense: bool):
        if dense:
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
            return o.transpose(1, 2).contiguous()
        from .attention import spark_attention_bthd

        return spark_attention_bthd(self.controller, q, k, v, self.layout, layer)

    def _out_quant(self, o_seg):
        # o_seg [P, Nloc, Hp, D]: row m of the output projection's input is the P segments
        P, M, hp, D = o_seg.shape
        q = torch.empty((M, P * hp * D), device=self.device, dtype=FP8_DTYPE)
        s = torch.empty((M, 1), device=self.device, dtype=torch.float32)
        _lib.call("sb_fp8_quantize_segments", o_seg.data_ptr(), M, P * hp * D, hp * D, M * hp * D, q.data_ptr(),
                  s.data_ptr(), _stream(self.device))
        return q, s

    def _gelu_quant(self, h):
        M, K = h.shape
        q = torch.empty((M, K), device=self.device, dtype=FP8_DTYPE)
        s = torch.empty((M, 1), device=self.device, dtype=torch.float32)
        _lib.call("sb_fp8_gelu_quantize_rows", h.data_ptr(), _lib.BF16, M, K, q.data_ptr(), s.data_ptr(),
                  _stream(self.device))
        return q, s

    def _exchange(self):
        """Brackets one exchange with CUDA events on the current stream when
        exchange_events is a list (a no-op context otherwise)."""
        import contextlib

        if self.exchange_events is None or self.world == 1:
            return contextlib.nullcontext()
        events = self.exchange_events
        stream = torch.cuda.current_stream(self.device)

        @contextlib.contextmanager
        def timed():
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            yield
            e1.record(stream)
            events.append((e0, e1))

        return timed()

    def modulation(self, t: float):
        temb = F.silu(timestep_embedding(t, self.cfg.t_dim, self.device))
        return [(blk["ada"] @ temb).view(6, self.cfg.hidden).contiguous() for blk in self.blocks]

    def step(self, x: torch.Tensor, t: float, *, dense: bool) -> torch.Tensor:
        """One denoise evaluation of the stack on this rank's tokens x [Nloc, hidden] bf16,
        updated in place."""
        if x.shape != (self.local, self.cfg.hidden) or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError(f"x must be contiguous bf16 [{self.local}, {self.cfg.hidden}]")
        for layer, (blk, mod) in enumerate(zip(self.blocks, self.modulation(t))):
            shift1, scale1, gate1, shift2, scale2, gate2 = mod
            hq, hs = self._norm_quant(x, shift1, scale1)
            if self.peer is not None:
                self._qkv_producer_peers(hq, hs, blk)
                self.peer.barrier()
                qh, kh, vh = (t_.reshape(-1, self.hp, self.cfg.head_dim).unsqueeze(0) for t_ in self.peer.views)
            else:
                if self.fused_producer:
                    q, k, v = self._qkv_producer(hq, hs, blk)
                else:
                    qkv = fp8_gemm(hq, hs, *blk["qkv"])
                    q, k, v = self._qkv_rope(qkv, blk)
                    del qkv
                with self._exchange():
                    qh, kh, vh = (exchange_to_heads(t_, self.group).unsqueeze(0) for t_ in (q, k, v))
                del q, k, v
            o = self._attention(qh, kh, vh, layer, dense)
            del qh, kh, vh
            with self._exchange():
                o_seg = exchange_to_tokens(o[0], self.world, self.group)
            oq, os_ = self._out_quant(o_seg)
            del o_seg
            self._gemm_residual(oq, os_, blk["out"], x, gate1)
            hq, hs = self._norm_quant(x, shift2, scale2)
            f = fp8_gemm(hq, hs, *blk["up"])
            fq, fs = self._gelu_quant(f)
            del f
            self._gemm_residual(fq, fs, blk["down"], x, gate2)
        return x


def reference_block_math(x, blk, mod, cfg: DiTConfig, coords, inv_freq, axis, attention):
    """fp32 torch restatement of one block on one rank (P = 1) with the same e4m3 activation
    and weight quantisation, for the tests."""
    from .fp8_linear import quantize_rows_reference

    def deq(w):
        return w[0].float() * w[1].reshape(-1, 1)

    def lin(h, w):
        hq, hs = quantize_rows_reference(h)
        return (hq.float() * hs) @ deq(w).T

    def norm_mod(h, shift, scale):
        h = h.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + cfg.eps)
        return h * (1 + scale) + shift

    shift1, scale1, gate1, shift2, scale2, gate2 = mod
    M = x.shape[0]
    qkv = lin(norm_mod(x, shift1, scale1), blk["qkv"]).to(torch.bfloat16).float().view(M, 3, cfg.heads, cfg.head_dim)
    ang = coords[:, axis.long()].float() * inv_freq  # [M, D/2]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

    def norm_rope(t_, w):
        t_ = t_ * torch.rsqrt(t_.pow(2).mean(-1, keepdim=True) + cfg.eps) * w
        a, b = t_[..., 0::2], t_[..., 1::2]
        out = torch.empty_like(t_)
        out[..., 0::2] = a * cos - b * sin
        out[..., 1::2] = a * sin + b * cos
        return out.to(torch.bfloat16)

    q = norm_rope(qkv[:, 0], blk["norm_q"])
    k = norm_rope(qkv[:, 1], blk["norm_k"])
    v = qkv[:, 2].to(torch.bfloat16)
    o = attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0))[0].reshape(M, -1)
    x = x.float() + gate1 * lin(o.float(), blk["out"])
    x = x.to(torch.bfloat16).float()
    f = lin(norm_mod(x, shift2, scale2), blk["up"]).to(torch.bfloat16).float()
    x = x + gate2 * lin(F.gelu(f), blk["down"])
    return x.to(torch.bfloat16)

"""e4m3 linears on the B200 tensor cores, with the module API of
h3_sparse_attention/fp8_linear.py (`quantize_rows`, `quantize_tensor`, `swiglu_quantize`,
`swiglu_quantize_tensor`, `Fp8Linear`, `forward_qkv_shared`, `Fp8SwiGLUFeedForward`,
`Fp8AttnProcessor`, `convert_linear_to_fp8`, `install_fp8`).

Scale granularity is per-token activation x per-output-channel weight on every card: the
tcgen05 GEMM in libsparkh3b200.so applies both scale vectors in its epilogue, so the
reference's sm100 switch to per-tensor scales (fp8_linear.py:50-62, 147-156, which exists
only because the library's rowwise-scaled GEMM was slow there) has nothing to buy here.
The per-tensor quantisers stay available and the GEMM accepts a one-element scale on
either side.

Weights are quantised once, at conversion, with the reference's own per-channel recipe
(fp8_linear.py:269-278): scale = max(absmax_row / 448, 1e-12) in fp32, codes =
e4m3(weight / bf16(scale)).  That one-time setup runs as plain torch on whatever device
holds the weight; every per-call operation (activation quantisation, SwiGLU fusion, GEMM)
runs in the CUDA library and fails loudly without it.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .ops import _dtype_code, _require_cuda, _stream

FP8_DTYPE = torch.float8_e4m3fn
FP8_MAX = 448.0
MIN_WIDTH = 4096
SKIP_END_BLOCKS = 0


def _rows(x: torch.Tensor) -> torch.Tensor:
    if x.dim() != 2:
        raise ValueError(f"expected [M, K], got {tuple(x.shape)}")
    return x.contiguous()


def quantize_rows(x: torch.Tensor):
    """bf16/fp32 [M, K] -> (e4m3 [M, K], fp32 scale [M, 1]): one absmax per row
    (fp8_linear.py:118-125)."""
    x = _rows(x)
    device = _require_cuda(x)
    M, K = x.shape
    y = torch.empty((M, K), device=device, dtype=FP8_DTYPE)
    scale = torch.empty((M, 1), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        _lib.call("sb_fp8_quantize_rows", x.data_ptr(), _dtype_code(x), M, K, y.data_ptr(), scale.data_ptr(),
                  _stream(device))
    return y, scale


def quantize_rows_reference(x: torch.Tensor):
    """The eager spelling of quantize_rows (fp8_linear.py:141-144), for the tests."""
    scale = (x.float().abs().amax(dim=1, keepdim=True) / FP8_MAX).clamp_min(1e-12)
    return (x.float() / scale).to(FP8_DTYPE), scale


def swiglu_quantize(h: torch.Tensor):
    """[M, 2K] projection output -> quantize_rows(a * silu(gate)) with a, gate = h.chunk(2),
    without writing the activation (fp8_linear.py:128-138)."""
    h = _rows(h)
    device = _require_cuda(h)
    M, K2 = h.shape
    K = K2 // 2
    y = torch.empty((M, K), device=device, dtype=FP8_DTYPE)
    scale = torch.empty((M, 1), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        _lib.call("sb_fp8_swiglu_quantize_rows", h.data_ptr(), _dtype_code(h), M, K, y.data_ptr(), scale.data_ptr(),
                  _stream(device))
    return y, scale


def quantize_tensor(x: torch.Tensor):
    """bf16/fp32 [M, K] -> (e4m3 [M, K], fp32 scale [1, 1]): one absmax for the tensor, the
    scale never leaves the device (fp8_linear.py:201-214)."""
    x = _rows(x)
    device = _require_cuda(x)
    y = torch.empty(x.shape, device=device, dtype=FP8_DTYPE)
    scale = torch.empty((1, 1), device=device, dtype=torch.float32)
    workspace = torch.empty(1, device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        _lib.call("sb_fp8_quantize_tensor", x.data_ptr(), _dtype_code(x), x.numel(), y.data_ptr(), scale.data_ptr(),
                  workspace.data_ptr(), _stream(device))
    return y, scale


def quantize_tensor_reference(x: torch.Tensor):
    """The eager spelling of quantize_tensor (fp8_linear.py:217-220), for the tests."""
    scale = (x.float().abs().amax() / FP8_MAX).clamp_min(1e-12).reshape(1, 1)
    return (x.float() / scale).to(FP8_DTYPE), scale


def swiglu_quantize_tensor(h: torch.Tensor):
    """[M, 2K] projection output -> per-tensor quantised bf16(a * silu(gate))
    (fp8_linear.py:223-239)."""
    h = _rows(h)
    device = _require_cuda(h)
    M, K2 = h.shape
    act = torch.empty((M, K2 // 2), device=device, dtype=torch.bfloat16)
    with torch.cuda.device(device):
        _lib.call("sb_fp8_swiglu", h.data_ptr(), _dtype_code(h), M, K2 // 2, act.data_ptr(), _stream(device))
    return quantize_tensor(act)


def quantize_activation(x: torch.Tensor):
    """What the GEMM callers use: per-token scales (the GEMM epilogue applies them)."""
    return quantize_rows(x)


def swiglu_quantize_activation(h: torch.Tensor):
    return swiglu_quantize(h)


def fp8_gemm(a_fp8: torch.Tensor, a_scale: torch.Tensor, b_fp8: torch.Tensor, b_scale: torch.Tensor,
             bias: torch.Tensor | None = None, out: torch.Tensor | None = None, num_ctas: int = 0) -> torch.Tensor:
    """bf16 [M, N] = (a_fp8 [M, K] . b_fp8 [N, K]^T) * a_scale * b_scale (+ bias).  Each scale
    holds one value per row of its operand, or a single value for the whole operand."""
    a_fp8, b_fp8 = a_fp8.contiguous(), b_fp8.contiguous()
    device = _require_cuda(a_fp8, b_fp8, a_scale.contiguous(), b_scale.contiguous(), bias, out)
    if a_fp8.dtype != FP8_DTYPE or b_fp8.dtype != FP8_DTYPE:
        raise TypeError("fp8_gemm takes float8_e4m3fn operands")
    M, K = a_fp8.shape
    N = b_fp8.shape[0]
    if b_fp8.shape[1] != K:
        raise ValueError(f"A [M, K] and B [N, K] must share K: {tuple(a_fp8.shape)} vs {tuple(b_fp8.shape)}")
    scales = []
    for scale, rows, name in ((a_scale, M, "a_scale"), (b_scale, N, "b_scale")):
        if scale.dtype != torch.float32:
            raise TypeError(f"{name} must be float32")
        if scale.numel() not in (1, rows):
            raise ValueError(f"{name} needs 1 or {rows} values, got {scale.numel()}")
        scales.append((scale.contiguous(), 1 if scale.numel() == rows and rows > 1 else 0))
    (a_scale, a_stride), (b_scale, b_stride) = scales
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
        if bias.numel() != N:
            raise ValueError(f"bias needs {N} values, got {bias.numel()}")
    if out is None:
        out = torch.empty((M, N), device=device, dtype=torch.bfloat16)
    with torch.cuda.device(device):
        _lib.call("sb_fp8_gemm", a_fp8.data_ptr(), a_scale.data_ptr(), a_stride, b_fp8.data_ptr(), b_scale.data_ptr(),
                  b_stride, M, N, K, None if bias is None else bias.data_ptr(), out.data_ptr(), num_ctas,
                  _stream(device))
    return out


def quantize_weight(weight: torch.Tensor):
    """Per-output-channel e4m3 weight (fp8_linear.py:269-278): (codes [N, K], scale [1, N])."""
    scale = (weight.abs().amax(dim=1, keepdim=True).float() / FP8_MAX).clamp_min(1e-12)
    codes = (weight / scale.to(weight.dtype)).to(FP8_DTYPE)
    return codes, scale.reshape(1, -1).contiguous()


class Fp8Linear(nn.Module):
    """A bias-optional Linear whose GEMM runs in e4m3 on the tensor cores (fp8_linear.py:252-293).

    The weight is quantised once, per output channel; the activation is quantised per token
    on every call, or by the caller (`forward_quantized`) when one activation feeds several
    of these.  Only the e4m3 copy, its scales and the bias are kept."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        codes, scale = quantize_weight(linear.weight.detach())
        self.register_buffer("weight_fp8", codes)
        self.register_buffer("weight_scale", scale)
        self.register_parameter("bias", linear.bias)
        self.in_features = linear.in_features
        self.out_features = linear.out_features

    def forward_quantized(self, x_fp8, x_scale, out_dtype=torch.bfloat16):
        """[M, K] e4m3 rows and their scales ([M, 1] per token or [1, 1]) -> [M, N]."""
        bias = None if self.bias is None else self.bias.detach()
        out = fp8_gemm(x_fp8, x_scale, self.weight_fp8, self.weight_scale, bias)
        return out if out_dtype == torch.bfloat16 else out.to(out_dtype)

    def forward(self, x):
        shape = x.shape
        rows = x.reshape(-1, shape[-1])
        out = self.forward_quantized(*quantize_activation(rows), out_dtype=rows.dtype)
        return out.reshape(*shape[:-1], -1)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def forward_qkv_shared(attn, hidden_states):
    """One quantisation of hidden_states feeds q/k/v when all three are Fp8Linear
    (fp8_linear.py:296-310); None otherwise, and the caller runs the plain projections."""
    projections = (attn.to_q, attn.to_k, attn.to_v)
    if not all(isinstance(p, Fp8Linear) for p in projections):
        return None
    rows = hidden_states.reshape(-1, hidden_states.shape[-1])
    x_fp8, x_scale = quantize_activation(rows)
    return tuple(p.forward_quantized(x_fp8, x_scale, out_dtype=hidden_states.dtype)
                 .reshape(*hidden_states.shape[:-1], -1) for p in projections)


class Fp8SwiGLUFeedForward(nn.Module):
    """FeedForward([SwiGLU, Dropout(0), Linear]) with both GEMMs in e4m3 and the SwiGLU fused
    into the quantisation of its output (fp8_linear.py:313-336); inference only."""

    def __init__(self, ff):
        super().__init__()
        swiglu, dropout, down = ff.net
        if getattr(dropout, "p", 0) != 0:
            raise ValueError("Fp8SwiGLUFeedForward fuses the activation with the quantisation; a live dropout "
                             "cannot be fused")
        self.proj = swiglu.proj
        self.down = down

    def forward(self, hidden_states):
        shape = hidden_states.shape
        h = self.proj(hidden_states.reshape(-1, shape[-1]))
        out = self.down.forward_quantized(*swiglu_quantize_activation(h), out_dtype=h.dtype)
        return out.reshape(*shape[:-1], -1)


class Fp8AttnProcessor:
    """Dense attention processor with one quantisation of hidden_states shared by q/k/v
    (fp8_linear.py:339-379).  Installed by `install_fp8` where all three projections are
    Fp8Linear; the sparse plugin adopts it as its dense path when installed afterwards."""

    _attention_backend = None
    _parallel_config = None

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        from .processor import apply_rotary_emb

        query, key, value = forward_qkv_shared(attn, hidden_states)
        query = attn.norm_q(query.unflatten(-1, (attn.heads, -1)))
        key = attn.norm_k(key.unflatten(-1, (attn.heads, -1)))
        value = value.unflatten(-1, (attn.heads, -1))
        if rotary_emb is not None:
            query = apply_rotary_emb(query, rotary_emb)
            key = apply_rotary_emb(key, rotary_emb)
        out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2),
                                             attn_mask=attention_mask)
        hidden_states = out.transpose(1, 2).flatten(2, 3).type_as(query)
        hidden_states = attn.to_out[0](hidden_states)
        return attn.to_out[1](hidden_states)


def _fuse_ff(block) -> bool:
    """block.ff -> Fp8SwiGLUFeedForward when both of its GEMMs became Fp8Linear
    (fp8_linear.py:382-395)."""
    ff = getattr(block, "ff", None)
    net = getattr(ff, "net", None)
    if net is None or len(net) != 3:
        return False
    swiglu, dropout, down = net
    if not (isinstance(getattr(swiglu, "proj", None), Fp8Linear) and isinstance(down, Fp8Linear)
            and getattr(dropout, "p", 0) == 0):
        return False
    block.ff = Fp8SwiGLUFeedForward(ff)
    return True


def convert_linear_to_fp8(model, min_width=MIN_WIDTH, skip_end_blocks=SKIP_END_BLOCKS):
    """Swap the Linears at least `min_width` wide on both sides inside
    model.transformer_blocks for Fp8Linear, in place, and fuse each converted block's SwiGLU
    FeedForward (fp8_linear.py:398-427).  `skip_end_blocks` keeps the first and last N blocks
    in bf16.  Returns how many Linears were swapped."""
    blocks = getattr(model, "transformer_blocks", None)
    if not blocks:
        raise ValueError("convert_linear_to_fp8 expects a model with a non-empty `transformer_blocks` ModuleList")
    swapped = 0
    for index, block in enumerate(blocks):
        if index < skip_end_blocks or index >= len(blocks) - skip_end_blocks:
            continue
        for parent in list(block.modules()):
            for name, child in list(parent.named_children()):
                if not isinstance(child, nn.Linear):
                    continue
                if child.in_features < min_width or child.out_features < min_width:
                    continue
                setattr(parent, name, Fp8Linear(child).to(child.weight.device))
                swapped += 1
        _fuse_ff(block)
    return swapped


def install_fp8(pipe_or_transformer, min_width=MIN_WIDTH, skip_end_blocks=SKIP_END_BLOCKS):
    """Convert a pipeline's (or a transformer's) wide block Linears, fuse the FeedForwards and
    install the shared-qkv processor on every converted attention (fp8_linear.py:430-447).
    Call after the weights are loaded and before the sparse-attention plugin.  Returns how
    many Linears were quantised."""
    transformer = getattr(pipe_or_transformer, "transformer", pipe_or_transformer)
    swapped = convert_linear_to_fp8(transformer, min_width=min_width, skip_end_blocks=skip_end_blocks)
    for block in transformer.transformer_blocks:
        attn = getattr(block, "attn", None)
        if (attn is not None and not getattr(attn, "fused_projections", False)
                and all(isinstance(getattr(attn, name, None), Fp8Linear) for name in ("to_q", "to_k", "to_v"))):
            attn.set_processor(Fp8AttnProcessor())
    return swapped

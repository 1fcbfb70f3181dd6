"""fp8 linears: the reference's own test cases (h3_sparse_attention tests/test_fp8_linear.py)
restated against the B200 library, plus the config-3 parity bar (relative Frobenius error
against a GEMM of the dequantised operands) at the full M = 124,992 rows."""
from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from spark_h3_b200.fp8_linear import (
    Fp8AttnProcessor, Fp8Linear, Fp8SwiGLUFeedForward, convert_linear_to_fp8, fp8_gemm, forward_qkv_shared,
    install_fp8, quantize_rows, quantize_rows_reference, quantize_tensor, quantize_tensor_reference,
    quantize_weight, swiglu_quantize, swiglu_quantize_tensor)

REL_FROBENIUS = 3e-2  # the config-3 bar for fp8 linears


def rel_frobenius(actual, expected):
    return float((actual.float() - expected.float()).norm() / expected.float().norm())


def dequantised_reference(x_fp8, x_scale, w_fp8, w_scale, bias=None):
    """fp32 GEMM of the dequantised operands: what the e4m3 GEMM computes, exactly up to
    the accumulation order and the final bf16 rounding."""
    a = x_fp8.float() * x_scale.reshape(-1, 1).float()
    b = w_fp8.float() * w_scale.reshape(-1, 1).float()
    out = a @ b.T
    return out if bias is None else out + bias.float()


# ---------------------------------------------------------------- CPU (host logic)

class SwiGLU(nn.Module):
    """diffusers' SwiGLU: one projection to 2 x inner, value half first, gate half second."""

    def __init__(self, dim, inner):
        super().__init__()
        self.proj = nn.Linear(dim, inner * 2, bias=False)

    def forward(self, x):
        a, gate = self.proj(x).chunk(2, dim=-1)
        return a * F.silu(gate)


class FeedForward(nn.Module):
    def __init__(self, dim=16, inner=32):
        super().__init__()
        self.net = nn.ModuleList([SwiGLU(dim, inner), nn.Dropout(0.0), nn.Linear(inner, dim, bias=False)])

    def forward(self, x):
        for module in self.net:
            x = module(x)
        return x


def fake_model(num_blocks=10, width=16, narrow=4):
    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.wide = nn.Linear(width, width, bias=False)
            self.narrow = nn.Linear(narrow, width, bias=False)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer_blocks = nn.ModuleList(Block() for _ in range(num_blocks))
            self.context_embedder = nn.Linear(width, width, bias=False)  # wide, outside the blocks

    return Model()


def test_convert_scopes_to_transformer_blocks():
    model = fake_model()
    assert convert_linear_to_fp8(model, min_width=8, skip_end_blocks=2) == 6
    for index, block in enumerate(model.transformer_blocks):
        assert type(block.wide) is (nn.Linear if index < 2 or index >= 8 else Fp8Linear)
        assert type(block.narrow) is nn.Linear
    assert type(model.context_embedder) is nn.Linear


def test_convert_rejects_model_without_blocks():
    with pytest.raises(ValueError, match="transformer_blocks"):
        convert_linear_to_fp8(nn.Linear(16, 16))


def test_install_fp8_accepts_pipeline_or_transformer():
    class Pipe:
        def __init__(self):
            self.transformer = fake_model()

    pipe = Pipe()
    assert install_fp8(pipe, min_width=8, skip_end_blocks=2) == 6
    assert type(pipe.transformer.transformer_blocks[4].wide) is Fp8Linear
    assert install_fp8(fake_model(), min_width=8, skip_end_blocks=0) == 10


def test_convert_fuses_swiglu_feedforward():
    class FfModel(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer_blocks = nn.ModuleList(nn.Module() for _ in range(4))
            for block in self.transformer_blocks:
                block.ff = FeedForward()

    model = FfModel()
    convert_linear_to_fp8(model, min_width=8, skip_end_blocks=1)
    for index, block in enumerate(model.transformer_blocks):
        if index in (0, 3):
            assert type(block.ff) is FeedForward
        else:
            assert type(block.ff) is Fp8SwiGLUFeedForward
            assert type(block.ff.proj) is Fp8Linear and type(block.ff.down) is Fp8Linear


def test_weight_quantisation_follows_the_reference_recipe():
    """Per output channel: fp32 scale = max(absmax / 448, 1e-12), codes = e4m3(w / bf16(scale))."""
    torch.manual_seed(3)
    w = (torch.randn(96, 80) * 0.02).to(torch.bfloat16)
    w[5] = 0  # an all-zero channel takes the 1e-12 floor
    codes, scale = quantize_weight(w)
    ref_scale = (w.abs().amax(dim=1, keepdim=True).float() / 448.0).clamp_min(1e-12)
    assert torch.equal(scale, ref_scale.reshape(1, -1))
    assert torch.equal(codes.view(torch.uint8), (w / ref_scale.to(w.dtype)).to(torch.float8_e4m3fn).view(torch.uint8))
    assert float(scale[0, 5]) == pytest.approx(1e-12)


def test_fp8_ops_refuse_cpu_tensors():
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_rows(torch.randn(4, 16))
    linear = Fp8Linear(nn.Linear(16, 16, bias=False))
    with pytest.raises(RuntimeError, match="CUDA"):
        linear(torch.randn(2, 16))


# ---------------------------------------------------------------- GPU

@pytest.mark.gpu
def test_quantize_rows_matches_reference(cuda_device):
    torch.manual_seed(21)
    for shape in ((517, 4099), (300, 4096), (1, 8)):
        x = torch.randn(*shape, device=cuda_device, dtype=torch.bfloat16) * 3
        y, scale = quantize_rows(x)
        y_ref, scale_ref = quantize_rows_reference(x)
        assert y.dtype == torch.float8_e4m3fn
        assert torch.equal(scale, scale_ref)
        assert torch.equal(y.view(torch.uint8), y_ref.view(torch.uint8))
    x = torch.randn(64, 520, device=cuda_device) * 100  # fp32 input, zero row
    x[7] = 0
    y, scale = quantize_rows(x)
    y_ref, scale_ref = quantize_rows_reference(x)
    assert torch.equal(scale, scale_ref) and torch.equal(y.view(torch.uint8), y_ref.view(torch.uint8))


@pytest.mark.gpu
def test_quantize_tensor_matches_reference(cuda_device):
    torch.manual_seed(22)
    for shape in ((517, 4099), (3, 5)):
        x = torch.randn(*shape, device=cuda_device, dtype=torch.bfloat16) * 3
        y, scale = quantize_tensor(x)
        y_ref, scale_ref = quantize_tensor_reference(x)
        assert scale.shape == (1, 1)
        assert torch.equal(scale, scale_ref)
        assert torch.equal(y.view(torch.uint8), y_ref.view(torch.uint8))


def assert_fp8_matches_activation(y, scale, activation):
    """Dequantisation lands within e4m3's own quantisation error of the true activation."""
    dequant = y.float() * scale
    ref = activation.float()
    assert F.cosine_similarity(dequant.flatten(), ref.flatten(), dim=0) > 0.999
    assert (dequant - ref).abs().max() <= ref.abs().max() * 2 ** -3


@pytest.mark.gpu
def test_swiglu_quantize_matches_fused_reference(cuda_device):
    torch.manual_seed(23)
    h = torch.randn(256, 4104 * 2, device=cuda_device, dtype=torch.bfloat16)
    y, scale = swiglu_quantize(h)
    a, gate = h.chunk(2, dim=-1)
    assert_fp8_matches_activation(y, scale, a * F.silu(gate))
    ref_scale = (a.float() * F.silu(gate.float())).abs().amax(dim=1, keepdim=True) / 448.0
    assert torch.allclose(scale, ref_scale.clamp_min(1e-12), rtol=2 ** -7)


@pytest.mark.gpu
def test_swiglu_quantize_tensor_matches_fused_reference(cuda_device):
    torch.manual_seed(24)
    h = torch.randn(256, 4104 * 2, device=cuda_device, dtype=torch.bfloat16)
    y, scale = swiglu_quantize_tensor(h)
    a, gate = h.chunk(2, dim=-1)
    act = a * F.silu(gate)
    assert_fp8_matches_activation(y, scale, act)
    ref_scale = (act.float().abs().amax() / 448.0).clamp_min(1e-12).reshape(1, 1)
    assert torch.allclose(scale, ref_scale, rtol=2 ** -7)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,bias", [(130, 64, 64, False), (300, 392, 4112, True), (1000, 1024, 512, False),
                                        (257, 520, 16, True)])
def test_fp8_gemm_matches_dequantised_reference(cuda_device, M, N, K, bias):
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.02
    b = torch.randn(N, device=cuda_device, dtype=torch.bfloat16) if bias else None
    x_fp8, x_scale = quantize_rows(x)
    w_fp8, w_scale = quantize_weight(w)
    out = fp8_gemm(x_fp8, x_scale, w_fp8, w_scale, b)
    ref = dequantised_reference(x_fp8, x_scale, w_fp8, w_scale, b)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    assert rel_frobenius(out, ref) <= 1e-2
    assert (out.float() - ref).abs().max() <= 2e-2 * ref.abs().max()


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,bias", [(512, 768, 1024, False), (4000, 2048, 4096, False), (1024, 1536, 4096, True)])
def test_fp8_gemm_matches_the_references_scaled_mm(cuda_device, M, N, K, bias):
    """The reference's own GEMM call on a B200 (fp8_linear.py:150-156, 280-287): per-tensor
    scales on both operands, `torch._scaled_mm(x, w.t(), scale_a, scale_b, out_dtype=bf16,
    use_fast_accum=True)`, then `out + bias` in bf16.  Both GEMMs sum exact e4m3 products in
    fp32 and round once to bf16, so they differ only where the summation order moves the fp32
    sum across a bf16 rounding boundary: at most one bf16 ulp, on a small share of the
    elements.  With a bias the reference rounds twice (the product, then the sum with the
    bias) where this GEMM rounds once, so each may be off by half an ulp of the product and
    of the sum; where the bias cancels the product, that bound is set by the product's
    magnitude, not the result's."""
    torch.manual_seed(M + 3 * N + K)
    x = (torch.randn(M, K, device=cuda_device) * torch.empty(M, 1, device=cuda_device).log_normal_(0.0, 0.5)
         ).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device) * 0.02).to(torch.bfloat16)
    b = torch.randn(N, device=cuda_device, dtype=torch.bfloat16) if bias else None
    x_fp8, x_scale = quantize_tensor(x)
    w_fp8, w_scale = quantize_tensor(w)
    ref = torch._scaled_mm(x_fp8, w_fp8.t(), scale_a=x_scale.reshape(()), scale_b=w_scale.reshape(()),
                           out_dtype=torch.bfloat16, use_fast_accum=True)
    if b is not None:
        ref = ref + b
    out = fp8_gemm(x_fp8, x_scale, w_fp8, w_scale, b)
    assert out.dtype == torch.bfloat16 and out.shape == ref.shape
    diff = (out.float() - ref.float()).abs()
    if b is None:
        assert bool((diff <= 2.0 ** -7 * ref.float().abs() + 1e-30).all()), float(diff.max())
        assert float((diff == 0).float().mean()) >= 0.98
        assert rel_frobenius(out, ref) <= 1e-3
    else:
        product = (ref.float() - b.float()).abs()
        bound = 2.0 ** -7 * (product + ref.float().abs()) + 1e-30
        assert bool((diff <= bound).all()), float((diff / bound).max())
        assert rel_frobenius(out, ref) <= 4e-3


@pytest.mark.gpu
def test_fp8_gemm_per_tensor_scales_and_persistent_grid(cuda_device):
    """Per-tensor scales on either side, and a grid smaller than the tile count (each CTA
    walks several tiles through both accumulators)."""
    torch.manual_seed(5)
    x = torch.randn(900, 1024, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(768, 1024, device=cuda_device, dtype=torch.bfloat16) * 0.02
    x_fp8, x_scale = quantize_tensor(x)
    w_fp8, w_scale = quantize_weight(w)
    ref = dequantised_reference(x_fp8, x_scale.expand(900, 1), w_fp8, w_scale)
    for ctas in (0, 1, 3, 7):
        out = fp8_gemm(x_fp8, x_scale, w_fp8, w_scale, num_ctas=ctas)
        assert rel_frobenius(out, ref) <= 1e-2
    w_fp8, w_scale = quantize_tensor(w)
    out = fp8_gemm(x_fp8, x_scale, w_fp8, w_scale)
    assert rel_frobenius(out, dequantised_reference(x_fp8, x_scale.expand(900, 1), w_fp8,
                                                    w_scale.expand(768, 1))) <= 1e-2


@pytest.mark.gpu
def test_fp8_linear_close_to_bf16(cuda_device):
    torch.manual_seed(25)
    linear = nn.Linear(5376, 7168, bias=False, device=cuda_device, dtype=torch.bfloat16)
    x = torch.randn(259, 5376, device=cuda_device, dtype=torch.bfloat16)
    expected = linear(x)
    actual = Fp8Linear(linear)(x)
    assert actual.shape == expected.shape
    assert F.cosine_similarity(expected.flatten().float(), actual.flatten().float(), dim=0) > 0.998


@pytest.mark.gpu
def test_forward_qkv_shared_bitwise_and_fallback(cuda_device):
    from types import SimpleNamespace

    torch.manual_seed(26)
    projections = [Fp8Linear(nn.Linear(64, 64, bias=False, device=cuda_device, dtype=torch.bfloat16))
                   for _ in range(3)]
    attn = SimpleNamespace(to_q=projections[0], to_k=projections[1], to_v=projections[2])
    x = torch.randn(1, 130, 64, device=cuda_device, dtype=torch.bfloat16)
    shared = forward_qkv_shared(attn, x)
    for projection, shared_out in zip(projections, shared):
        assert torch.equal(shared_out, projection(x))
    attn.to_k = nn.Linear(64, 64, bias=False, device=cuda_device, dtype=torch.bfloat16)
    assert forward_qkv_shared(attn, x) is None


@pytest.mark.gpu
def test_fused_feedforward_close_to_bf16(cuda_device):
    torch.manual_seed(27)
    ff = FeedForward(dim=5376, inner=14336).to(cuda_device, torch.bfloat16).eval()
    x = torch.randn(1, 259, 5376, device=cuda_device, dtype=torch.bfloat16) * 3
    with torch.no_grad():
        expected = ff(x)
        block = nn.Module()
        block.ff = ff
        model = nn.Module()
        model.transformer_blocks = nn.ModuleList([block])
        convert_linear_to_fp8(model, min_width=8, skip_end_blocks=0)
        assert type(block.ff) is Fp8SwiGLUFeedForward
        actual = block.ff(x)
    assert F.cosine_similarity(expected.flatten().float(), actual.flatten().float(), dim=0) > 0.995


@pytest.mark.gpu
def test_install_fp8_attention_processor(cuda_device):
    from test_gpu_plugin import TinyAttention

    class DenseProcessor:
        def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
            q, k, v = (p(hidden_states).unflatten(-1, (attn.heads, -1)).transpose(1, 2)
                       for p in (attn.to_q, attn.to_k, attn.to_v))
            out = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).flatten(2, 3)
            return attn.to_out[1](attn.to_out[0](out))

    torch.manual_seed(28)
    attn = TinyAttention(hidden=128, heads=1).to(cuda_device, torch.bfloat16).eval()
    attn.set_processor(DenseProcessor())
    model = nn.Module()
    model.transformer_blocks = nn.ModuleList([nn.Module()])
    model.transformer_blocks[0].attn = attn
    x = torch.randn(1, 259, 128, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        expected = attn(x)
        assert install_fp8(model, min_width=8, skip_end_blocks=0) == 3
        assert type(attn.get_processor()) is Fp8AttnProcessor
        actual = attn(x)
    assert F.cosine_similarity(expected.flatten().float(), actual.flatten().float(), dim=0) > 0.995


@pytest.mark.gpu
@pytest.mark.parametrize("N", [12288, 4096, 16384])
def test_config3_full_size_rel_frobenius(cuda_device, N):
    """Config 3 at full size: X [124992, 4096] ~ N(0,1) x LogNormal(0, 0.5) per token,
    W ~ N(0, 0.02).  The e4m3 linear against a bf16 GEMM of the dequantised operands, and the
    GEMM itself against an fp32 GEMM of the same operands on sampled rows."""
    M, K = 124992, 4096
    g = torch.Generator(device=cuda_device).manual_seed(N)
    x = (torch.randn(M, K, device=cuda_device, generator=g)
         * torch.empty(M, 1, device=cuda_device).log_normal_(0.0, 0.5, generator=g)).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    x_fp8, x_scale = quantize_rows(x)
    w_fp8, w_scale = quantize_weight(w)
    out = fp8_gemm(x_fp8, x_scale, w_fp8, w_scale)
    del x
    rows = torch.cat([torch.randint(0, M, (2048,), device=cuda_device, generator=g),
                      torch.arange(M - 192, M, device=cuda_device)])
    a = (x_fp8[rows].float() * x_scale[rows]).to(torch.bfloat16)
    b = (w_fp8.float() * w_scale.reshape(-1, 1)).to(torch.bfloat16)
    assert rel_frobenius(out[rows], a @ b.T) <= REL_FROBENIUS
    exact = dequantised_reference(x_fp8[rows], x_scale[rows], w_fp8, w_scale)
    assert rel_frobenius(out[rows], exact) <= 1e-2
    assert torch.isfinite(out).all()

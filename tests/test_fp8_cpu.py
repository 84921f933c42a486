"""CPU oracle of the block-scaled FP8 recipe: power-of-two scales, E4M3 bytes, dequant; MXFP4 and
per-axis FP8 fake quantisation."""

import pytest
import torch

from saint_llm_b200.ops import fp8
from saint_llm_b200.ops.quant import E4M3_MAX, pow2_scale


def test_pow2_scale_is_exact_ceiling():
    amax = torch.tensor([0.0, 448.0, 448.0 * (1 + 2**-23), 224.0, 1.0, 448 * 2.0**-10])
    s = pow2_scale(amax)
    assert s.tolist() == [1.0, 1.0, 2.0, 0.5, 2.0**-8, 2.0**-10]
    # the scaled amax never exceeds the E4M3 range and halving the scale would
    assert ((amax / s) <= E4M3_MAX).all()
    assert ((amax[1:] / (s[1:] / 2)) > E4M3_MAX).all()


def test_oracle_roundtrip_and_gemm():
    torch.manual_seed(0)
    x = torch.randn(96, 256) * 3
    w = torch.randn(128, 256) * 0.02
    a, b = fp8.quantize_rows(x), fp8.quantize_blocks(w)
    assert a.q.dtype == torch.uint8 and a.scale.shape == (96, 2) and b.scale.shape == (1, 2)
    assert ((a.dequantize() - x).abs() <= x.abs() * 2**-3 + 1e-6).all()  # E4M3 keeps 3 mantissa bits
    y = fp8.gemm(a, b)
    assert y.dtype == torch.bfloat16 and y.shape == (96, 128)
    ref = x @ w.t()
    assert (y.float() - ref).norm() < 0.06 * ref.norm()
    z = fp8.linear(x.reshape(2, 48, 256), w)
    assert z.shape == (2, 48, 128)


def test_fp8_block_quant_properties():
    """Row (1 x 128) and block (128 x 128) quantisation: power-of-two scales, every value in
    range, small relative error, zero blocks exact, and shape checks."""
    from saint_llm_b200.ops.quant import (
        E4M3_MAX,
        dequantize_fp8_blocks,
        dequantize_fp8_rows,
        quantize_fp8_blocks,
        quantize_fp8_rows,
    )

    torch.manual_seed(0)
    x = torch.randn(4, 256) * torch.logspace(-3, 3, 4)[:, None]
    x[1, :128] = 0.0
    q, s = quantize_fp8_rows(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (4, 2)
    assert torch.equal(torch.frexp(s)[0], torch.full_like(s, 0.5))  # powers of two
    assert (q.float().abs() <= E4M3_MAX).all()
    back = dequantize_fp8_rows(q, s)
    assert torch.equal(back[1, :128], torch.zeros(128))
    rel = (back - x).abs().sum() / x.abs().sum()
    assert rel < 0.05
    w = torch.randn(256, 384)
    qw, sw = quantize_fp8_blocks(w)
    assert sw.shape == (2, 3)
    torch.testing.assert_close(dequantize_fp8_blocks(qw, sw), w, rtol=0.07, atol=0.02)
    with pytest.raises(ValueError):
        quantize_fp8_rows(torch.randn(2, 100))
    with pytest.raises(ValueError):
        quantize_fp8_blocks(torch.randn(100, 128))


def test_mxfp4_fake_quant_grid_and_straight_through():
    """MXFP4: every dequantised value is an E2M1 level times its block's power-of-two scale,
    the block maximum maps to at most 6, and the backward passes gradients straight through."""
    from saint_llm_b200.ops.quant import FP4_E2M1_LEVELS, cast_to_fp4_mx, fake_quant_fp4_mx

    torch.manual_seed(1)
    x = torch.randn(3, 64) * 5
    deq, scale = cast_to_fp4_mx(x, block_size=32)
    assert scale.shape == (3, 2)
    blocks = (deq.view(3, 2, 32) / scale[..., None]).abs()
    levels = FP4_E2M1_LEVELS
    assert torch.isin(blocks, levels).all()
    assert ((x.view(3, 2, 32).abs().amax(-1) / scale) <= 6.0 + 1e-6).all()
    xr = x.clone().requires_grad_(True)
    y = fake_quant_fp4_mx(xr)
    y.sum().backward()
    assert torch.equal(xr.grad, torch.ones_like(x)) and torch.equal(y.detach(), deq)
    with pytest.raises(ValueError):
        cast_to_fp4_mx(torch.randn(2, 40), block_size=32)


def test_fp8_per_axis_cast_and_fake_quant():
    from saint_llm_b200.ops.quant import Fp8Format, cast_to_fp8, dequant_from_fp8, fake_quant_fp8

    torch.manual_seed(2)
    x = torch.randn(5, 7) * torch.arange(1, 6)[:, None]
    for fmt in (Fp8Format.E4M3, Fp8Format.E5M2):
        q, s = cast_to_fp8(x, fmt, axis=0)
        assert s.shape == (5, 1) and q.dtype == fmt.dtype
        assert torch.allclose(x.abs().amax(1, keepdim=True) / s, torch.full((5, 1), fmt.fmax))
        back = dequant_from_fp8(q, s)
        assert ((back - x).abs() <= x.abs().amax(1, keepdim=True) * (0.07 if fmt is Fp8Format.E4M3 else 0.13)).all()
    xr = x.clone().requires_grad_(True)
    fake_quant_fp8(xr).sum().backward()
    assert torch.equal(xr.grad, torch.ones_like(x))


@pytest.mark.parametrize("mode", ["fp8", "fp4"])
def test_qat_linears_track_the_plain_linear(mode):
    """The QAT linears of the factory (eager CPU path) stay close to the plain linear they are
    built from, pass gradients to input, weight and bias, and keep the layer's shape / repr."""
    from torch import nn

    from saint_llm_b200.models.linear import Fp4Linear, Fp8Linear, make_linear_factory

    torch.manual_seed(3)
    base = nn.Linear(64, 32)
    layer = (Fp8Linear if mode == "fp8" else Fp4Linear).from_linear(base)
    x = torch.randn(5, 64, requires_grad=True)
    y, ref = layer(x), base(x)
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel < (0.05 if mode == "fp8" else 0.25), rel
    y.sum().backward()
    assert x.grad is not None and layer.weight.grad is not None and layer.bias.grad is not None
    assert "in_features=64" in repr(layer)
    made = make_linear_factory(mode)(64, 32, bias=False)
    assert made.bias is None and made.weight.shape == (32, 64)
    with pytest.raises(ValueError):
        make_linear_factory("int4")  # type: ignore[arg-type]
    if mode == "fp4":
        with pytest.raises(ValueError):
            Fp4Linear(50, 8)

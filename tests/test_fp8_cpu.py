"""CPU oracle of the block-scaled FP8 recipe: power-of-two scales, E4M3 bytes, dequant."""

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

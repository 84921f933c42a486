"""FP8 / MXFP4 quantisation: eager references (the oracle) and native entry points.

Eager semantics follow the reference (``kernels/quant/reference.py:32-134``,
``kernels/quant/fp4.py:28-131``):

* FP8 absmax: ``s = max(amax/fmax, tiny)`` per tensor or per kept axis,
  ``q = clamp(x/s, -fmax, fmax).to(fp8)`` (round-to-nearest-even), ``x_hat = q*s``.
* MXFP4: blocks of ``block_size`` along an axis, scale ``2^ceil(log2(amax/6))``
  round-tripped through E8M0, elements rounded to the nearest E2M1 magnitude
  ``{0, .5, 1, 1.5, 2, 3, 4, 6}`` with ties resolved toward the lower level (the
  first minimum of the distance).
* ``fake_quant_*`` use the straight-through estimator ``x + (deq - x).detach()``.

Block-scaled FP8 for the tensor cores (``quantize_fp8_blocks``) is this framework's
training recipe: 1x128 activation blocks and 128x128 weight blocks with power-of-two
(UE8M0) scales, so the scales can be applied by the block-scaled MMA itself.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum

import torch
from torch import Tensor


class Fp8Format(Enum):
    E4M3 = "e4m3"
    E5M2 = "e5m2"

    @property
    def dtype(self) -> torch.dtype:
        return torch.float8_e4m3fn if self is Fp8Format.E4M3 else torch.float8_e5m2

    @property
    def fmax(self) -> float:
        return float(torch.finfo(self.dtype).max)


@dataclass(frozen=True)
class _Reduce:
    dims: tuple[int, ...]
    keepdim: bool


def _reduce_plan(ndim: int, axis: int | None) -> _Reduce:
    if axis is None:
        return _Reduce(tuple(range(ndim)), False)
    keep = axis % ndim
    return _Reduce(tuple(d for d in range(ndim) if d != keep), True)


def cast_to_fp8(x: Tensor, fmt: Fp8Format = Fp8Format.E4M3, *, axis: int | None = None,
                scale: Tensor | None = None) -> tuple[Tensor, Tensor]:
    plan = _reduce_plan(x.ndim, axis)
    if scale is None:
        amax = x.detach().abs().to(torch.float32)
        if plan.dims:
            amax = amax.amax(dim=plan.dims, keepdim=plan.keepdim)
        scale = (amax / fmt.fmax).clamp(min=torch.finfo(torch.float32).tiny)
    elif axis is not None and scale.ndim != x.ndim:
        keep = axis % x.ndim
        scale = scale.reshape([x.shape[keep] if d == keep else 1 for d in range(x.ndim)])
    q = (x.to(torch.float32) / scale).clamp(-fmt.fmax, fmt.fmax).to(fmt.dtype)
    return q, scale


def dequant_from_fp8(q: Tensor, scale: Tensor) -> Tensor:
    return q.to(torch.float32) * scale


def fake_quant_fp8(x: Tensor, fmt: Fp8Format = Fp8Format.E4M3, *, axis: int | None = None) -> Tensor:
    q, s = cast_to_fp8(x, fmt=fmt, axis=axis)
    return x + (dequant_from_fp8(q, s).to(x.dtype) - x).detach()


FP4_E2M1_FMAX = 6.0
FP4_E2M1_LEVELS = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)


def _round_e2m1(v: Tensor) -> Tensor:
    levels = FP4_E2M1_LEVELS.to(device=v.device, dtype=v.dtype)
    mag = v.abs().clamp(max=FP4_E2M1_FMAX)
    nearest = (mag.unsqueeze(-1) - levels).abs().argmin(dim=-1)
    return torch.sign(v) * levels[nearest]


def _e8m0_scale(amax: Tensor) -> Tensor:
    raw = (amax / FP4_E2M1_FMAX).clamp(min=torch.finfo(torch.float32).tiny)
    p2 = torch.pow(torch.tensor(2.0, dtype=torch.float32, device=amax.device), torch.ceil(torch.log2(raw)))
    return p2.to(torch.float8_e8m0fnu).to(torch.float32)


def cast_to_fp4_mx(x: Tensor, *, block_size: int = 32, axis: int = -1) -> tuple[Tensor, Tensor]:
    ax = axis % x.ndim
    if x.shape[ax] % block_size:
        raise ValueError(f"axis size {x.shape[ax]} must be a multiple of block_size {block_size}")
    xm = x.movedim(ax, -1)
    lead = xm.shape[:-1]
    nb = xm.shape[-1] // block_size
    blocks = xm.reshape(*lead, nb, block_size).to(torch.float32)
    scale = _e8m0_scale(blocks.abs().amax(dim=-1, keepdim=True))
    deq = (_round_e2m1(blocks / scale) * scale).reshape(*lead, nb * block_size)
    return deq.movedim(-1, ax).contiguous(), scale.squeeze(-1).movedim(-1, ax).contiguous()


def dequant_from_fp4_mx(fp4: Tensor, scale: Tensor) -> Tensor:
    del scale
    return fp4.to(torch.float32)


def fake_quant_fp4_mx(x: Tensor, *, block_size: int = 32, axis: int = -1) -> Tensor:
    q, _ = cast_to_fp4_mx(x, block_size=block_size, axis=axis)
    return x + (q.to(x.dtype) - x).detach()


# ---------------------------------------------------------------------------------
# Block-scaled FP8 (UE8M0 scales) -- eager reference of the native quant kernels.
# ---------------------------------------------------------------------------------
E4M3_MAX = 448.0


def pow2_scale(amax: Tensor, fmax: float = E4M3_MAX) -> Tensor:
    """Smallest power of two s with amax / s <= fmax (amax == 0 -> 1)."""
    raw = torch.where(amax > 0, amax.float() / fmax, torch.ones_like(amax, dtype=torch.float32))
    # exact ceil(log2(raw)) from the binary exponent (log2 rounding can land on an integer
    # just below the true value): raw = m * 2^e, m in [0.5, 1)
    m, e = torch.frexp(raw)
    e = torch.where(m == 0.5, e - 1, e).clamp(-126, 126)
    return torch.ldexp(torch.ones_like(raw), e)


def quantize_fp8_rows(x: Tensor, block: int = 128) -> tuple[Tensor, Tensor]:
    """1 x ``block`` activation quantisation of a (M, K) tensor -> (fp8 (M,K), scale (M, K/block))."""
    m, k = x.shape
    if k % block:
        raise ValueError("K must be a multiple of the block")
    xb = x.float().reshape(m, k // block, block)
    s = pow2_scale(xb.abs().amax(-1))
    q = (xb / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(m, k), s


def quantize_fp8_blocks(w: Tensor, block: int = 128) -> tuple[Tensor, Tensor]:
    """``block`` x ``block`` weight quantisation of a (N, K) tensor -> (fp8, scale (N/b, K/b))."""
    n, k = w.shape
    if n % block or k % block:
        raise ValueError("both dims must be multiples of the block")
    wb = w.float().reshape(n // block, block, k // block, block)
    s = pow2_scale(wb.abs().amax(dim=(1, 3)))
    q = (wb / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(n, k), s


def dequantize_fp8_rows(q: Tensor, s: Tensor, block: int = 128) -> Tensor:
    m, k = q.shape
    return (q.float().reshape(m, k // block, block) * s[..., None]).reshape(m, k)


def dequantize_fp8_blocks(q: Tensor, s: Tensor, block: int = 128) -> Tensor:
    n, k = q.shape
    return (q.float().reshape(n // block, block, k // block, block) * s[:, None, :, None]).reshape(n, k)


__all__ = [
    "E4M3_MAX",
    "FP4_E2M1_FMAX",
    "FP4_E2M1_LEVELS",
    "Fp8Format",
    "cast_to_fp4_mx",
    "cast_to_fp8",
    "dequant_from_fp4_mx",
    "dequant_from_fp8",
    "dequantize_fp8_blocks",
    "dequantize_fp8_rows",
    "fake_quant_fp4_mx",
    "fake_quant_fp8",
    "pow2_scale",
    "quantize_fp8_blocks",
    "quantize_fp8_rows",
]

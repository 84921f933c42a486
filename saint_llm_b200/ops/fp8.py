"""Block-scaled FP8 on the tensor cores: quantisation kernels and the tcgen05 GEMM.

``quantize_rows(x)`` quantises activations in 1 x 128 blocks, ``quantize_blocks(w)``
weights in 128 x 128 blocks; both give E4M3 values with power-of-two scales (the
smallest 2^e with amax / 2^e <= 448).  ``gemm(a, b)`` computes
``dequant(a) @ dequant(b)^T`` in bf16 with the block scales applied inside the MMA
(``tcgen05.mma kind::mxf8f6f4.block_scale``), so the operands stay FP8 all the way.

The reference quantises the same way in eager PyTorch (``kernels/quant/reference.py:32-134``)
and runs its real FP8 forward through ``torch._scaled_mm`` with rowwise / per-channel
scales (``kernels/fp8_gemm.py:24-101``).  On CPU (and under ``backend.eager_mode``) the
functions here run the PyTorch oracle of the same recipe: identical E4M3 bytes and scales,
an fp32 product of the dequantised operands.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from saint_llm_b200.ops import backend
from saint_llm_b200.ops.gemm import error_word
from saint_llm_b200.ops.quant import E4M3_MAX, pow2_scale

BLOCK = 128


@dataclass
class Fp8Operand:
    """E4M3 values (R, K) as bytes, fp32 block scales, and (native only) the scale-factor
    bytes in the layout the GEMM copies into tensor memory."""

    q: Tensor
    scale: Tensor
    sf: Tensor | None
    kind: str  # "rows" (scale (R, K/128)) or "blocks" (scale (R/128, K/128))

    @property
    def shape(self) -> torch.Size:
        return self.q.shape

    def dequantize(self) -> Tensor:
        r, k = self.q.shape
        v = self.q.view(torch.float8_e4m3fn).float()
        if self.kind == "rows":
            return (v.reshape(r, k // BLOCK, BLOCK) * self.scale[..., None]).reshape(r, k)
        return (v.reshape(r // BLOCK, BLOCK, k // BLOCK, BLOCK) * self.scale[:, None, :, None]).reshape(r, k)


def _oracle_rows(x: Tensor) -> Fp8Operand:
    m, k = x.shape
    xb = x.float().reshape(m, k // BLOCK, BLOCK)
    s = pow2_scale(xb.abs().amax(-1))
    q = (xb / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).reshape(m, k)
    return Fp8Operand(q.view(torch.uint8), s, None, "rows")


def _oracle_blocks(w: Tensor) -> Fp8Operand:
    n, k = w.shape
    wb = w.float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    s = pow2_scale(wb.abs().amax(dim=(1, 3)))
    q = (wb / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).reshape(n, k)
    return Fp8Operand(q.view(torch.uint8), s, None, "blocks")


def _check(t: Tensor, rows_mult: int) -> None:
    if t.dim() != 2 or t.shape[-1] % BLOCK or t.shape[0] % rows_mult:
        raise ValueError(f"FP8 operand {tuple(t.shape)} must be 2-D with K % 128 == 0"
                         + (" and rows % 128 == 0" if rows_mult > 1 else ""))


def quantize_rows(x: Tensor) -> Fp8Operand:
    """1 x 128 activation quantisation of (M, K)."""
    _check(x, 1)
    if not backend.native_for(x):
        return _oracle_rows(x)
    x = x.to(torch.bfloat16)
    if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.uint8, device=x.device)
    sf = torch.empty(backend.ext().fp8_sf_bytes(m, k), dtype=torch.uint8, device=x.device)
    scale = torch.empty((m, k // BLOCK), dtype=torch.float32, device=x.device)
    backend.ext().fp8_quant_rows(x, q, sf, scale)
    return Fp8Operand(q, scale, sf, "rows")


def quantize_blocks(w: Tensor) -> Fp8Operand:
    """128 x 128 weight quantisation of (N, K)."""
    _check(w, BLOCK)
    if not backend.native_for(w):
        return _oracle_blocks(w)
    w = w.to(torch.bfloat16)
    if w.stride(-1) != 1 or w.stride(0) % 8 or w.data_ptr() % 16:
        w = w.contiguous()
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.uint8, device=w.device)
    sf = torch.empty(backend.ext().fp8_sf_bytes(n, k), dtype=torch.uint8, device=w.device)
    scale = torch.empty((n // BLOCK, k // BLOCK), dtype=torch.float32, device=w.device)
    backend.ext().fp8_quant_blocks(w, q, sf, scale)
    return Fp8Operand(q, scale, sf, "blocks")


def gemm(a: Fp8Operand, b: Fp8Operand) -> Tensor:
    """bf16 (M, N) = dequant(a) @ dequant(b)^T; ``a`` from ``quantize_rows``, ``b`` from
    ``quantize_blocks`` (N % 128 == 0)."""
    if a.shape[1] != b.shape[1]:
        raise ValueError(f"K mismatch: {tuple(a.shape)} vs {tuple(b.shape)}")
    if a.sf is None or b.sf is None or not a.q.is_cuda or not backend.native_for(a.q):
        return (a.dequantize() @ b.dequantize().t()).to(torch.bfloat16)
    out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16, device=a.q.device)
    backend.ext().gemm_fp8(a.q, a.sf, b.q, b.sf, out, error_word(a.q.device))
    return out


def linear(x: Tensor, w: Tensor) -> Tensor:
    """``x @ w^T`` with the block-scaled FP8 recipe (x: (..., K), w: (N, K))."""
    k = x.shape[-1]
    y = gemm(quantize_rows(x.reshape(-1, k)), quantize_blocks(w))
    return y.reshape(*x.shape[:-1], w.shape[0])


__all__ = ["BLOCK", "Fp8Operand", "gemm", "linear", "quantize_blocks", "quantize_rows"]

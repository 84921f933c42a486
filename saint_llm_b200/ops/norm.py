"""RMSNorm and fused RoPE+RMSNorm on the native kernels (autograd-aware)."""

from __future__ import annotations

import torch
from torch import Tensor

from saint_llm_b200.ops import backend


def _bf16c(t: Tensor) -> Tensor:
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def _grad_to_param(weight: Tensor, dw: Tensor) -> Tensor | None:
    mg = getattr(weight, "main_grad", None)
    if mg is not None:
        mg.add_(dw)
        return None
    return dw.to(weight.dtype)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, eps: float) -> Tensor:  # type: ignore[override]
        xc = _bf16c(x)
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.numel() // xc.shape[-1], dtype=torch.float32, device=x.device)
        backend.ext().rmsnorm_fwd(xc, weight.float().contiguous(), y, rstd, float(eps))
        ctx.save_for_backward(xc, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        xc, weight, rstd = ctx.saved_tensors
        dx = torch.empty_like(xc)
        dw = backend.ext().rmsnorm_bwd(_bf16c(dy), xc, weight.float().contiguous(), rstd, dx)
        return dx, (_grad_to_param(weight, dw) if ctx.needs_input_grad[1] else None), None


def rms_norm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    return _RMSNormFn.apply(x, weight, eps)


class _RopeNormFn(torch.autograd.Function):
    """x: (T, H, hd) rows; cos/sin: (T, rd/2) fp32."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, cos: Tensor, sin: Tensor, rd: int, norm_first: bool,  # type: ignore[override]
                eps: float) -> Tensor:
        xc = _bf16c(x)
        heads = xc.shape[-2] if xc.dim() >= 3 else 1
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.numel() // xc.shape[-1], dtype=torch.float32, device=x.device)
        cs, sn = cos.float().contiguous(), sin.float().contiguous()
        backend.ext().rope_norm_fwd(xc, weight.float().contiguous(), cs, sn, y, rstd, heads, rd, norm_first,
                                    float(eps))
        ctx.save_for_backward(xc, weight, cs, sn, rstd)
        ctx.meta = (heads, rd, norm_first)
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        xc, weight, cs, sn, rstd = ctx.saved_tensors
        heads, rd, norm_first = ctx.meta
        dx = torch.empty_like(xc)
        dw = backend.ext().rope_norm_bwd(_bf16c(dy), xc, weight.float().contiguous(), cs, sn, rstd, dx, heads, rd,
                                         norm_first)
        return dx, (_grad_to_param(weight, dw) if ctx.needs_input_grad[1] else None), None, None, None, None, None


def rope_norm(x: Tensor, weight: Tensor, cos: Tensor, sin: Tensor, rope_dim: int, *, norm_first: bool,
              eps: float = 1e-6) -> Tensor:
    """x (T, H, hd) -> rope(norm(x)) if norm_first else norm(rope(x)); RoPE on the last rope_dim."""
    return _RopeNormFn.apply(x, weight, cos, sin, rope_dim, norm_first, eps)


__all__ = ["rms_norm", "rope_norm"]

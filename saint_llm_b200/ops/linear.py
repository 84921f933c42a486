"""Linear layers on the native GEMM, with fp32 gradient accumulation.

Forward ``y = x W^T (+ b)`` and backward ``dx = dy W`` run on the tcgen05 GEMM with
bf16 operands.  The weight gradient ``dW = dy^T x`` is written by the GEMM epilogue
straight into ``weight.main_grad`` (fp32, ``+=``) when the parameter carries one --
no bf16 rounding of gradients across micro-batches and no extra add kernel.  Without
``main_grad`` the gradient is returned to autograd in the parameter's dtype.

``fp8_linear`` applies the block-scaled FP8 recipe (1x128 activation / 128x128 weight
blocks, power-of-two scales): both operands are quantised by native kernels and the
product runs on the block-scaled FP8 tensor-core GEMM (``ops.fp8``); the backward is the
straight-through estimator in bf16, as in the reference (``kernels/fp8_gemm.py:71-83``).
The weight's FP8 copy is cached on the parameter (``ops.fp8.Fp8WeightCache``) and
re-quantised once per optimizer step, not once per micro-batch.
"""

from __future__ import annotations

import torch
from torch import Tensor

from saint_llm_b200.ops import fp8, gemm


def _bf16(t: Tensor) -> Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def accumulate_weight_grad(weight: Tensor, dy2: Tensor, x2: Tensor) -> Tensor | None:
    """dW = dy2^T @ x2 into weight.main_grad (returns None) or as a new tensor."""
    from saint_llm_b200.utils.profiling import phase

    mg = getattr(weight, "main_grad", None)
    with phase(f"wgrad.{dy2.shape[-1]}x{x2.shape[-1]}"):
        if mg is not None:
            gemm.gemm_nt(dy2.t(), x2.t(), out=mg, accumulate=True)
            return None
        return gemm.gemm_nt(dy2.t(), x2.t(), out_dtype=torch.float32).to(weight.dtype)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:  # type: ignore[override]
        k = x.shape[-1]
        x2 = _bf16(x.reshape(-1, k))
        y = gemm.gemm_nt(x2, _bf16(weight))
        if bias is not None:
            y = y + bias.to(y.dtype)
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.in_dtype = x.dtype
        return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, weight = ctx.saved_tensors
        n = weight.shape[0]
        dy2 = _bf16(dy.reshape(-1, n))
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm.gemm_nt(dy2, _bf16(weight).t()).reshape(*dy.shape[:-1], weight.shape[1])
            if ctx.in_dtype != torch.bfloat16:
                dx = dx.to(ctx.in_dtype)
        dw = accumulate_weight_grad(weight, dy2, x2) if ctx.needs_input_grad[1] else None
        db = dy2.float().sum(0).to(dy.dtype) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def linear(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    return _LinearFn.apply(x, weight, bias)


def fp8_shape_ok(in_features: int, out_features: int) -> bool:
    return in_features % 128 == 0 and out_features % 128 == 0


class _Fp8LinearFn(torch.autograd.Function):
    """Block-scaled FP8 forward (x: 1x128 blocks, W: 128x128 blocks), STE backward."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:  # type: ignore[override]
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        y = fp8.gemm(fp8.quantize_rows(x2), fp8.cached_weight(weight, "_fp8_cache", [weight]))
        if bias is not None:
            y = y + bias.to(y.dtype)
        ctx.save_for_backward(_bf16(x2), weight)
        ctx.has_bias = bias is not None
        return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, weight = ctx.saved_tensors
        dy2 = _bf16(dy.reshape(-1, weight.shape[0]))
        dx = gemm.gemm_nt(dy2, _bf16(weight).t()).reshape(*dy.shape[:-1], weight.shape[1])
        dw = accumulate_weight_grad(weight, dy2, x2) if ctx.needs_input_grad[1] else None
        db = dy2.float().sum(0).to(dy.dtype) if ctx.has_bias else None
        return dx, dw, db


def fp8_linear(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    return _Fp8LinearFn.apply(x, weight, bias)


class _FakeQuantFp4Fn(torch.autograd.Function):
    """MX FP4 straight-through fake quantisation in one native kernel (blocks of 32 along
    the last axis); the gradient passes through unchanged."""

    @staticmethod
    def forward(ctx, x: Tensor) -> Tensor:  # type: ignore[override]
        from saint_llm_b200.ops import backend

        xc = x.contiguous()
        out = torch.empty_like(xc)
        backend.ext().fake_quant_fp4(xc, out)
        return out.view_as(x)

    @staticmethod
    def backward(ctx, g: Tensor) -> Tensor:  # type: ignore[override]
        return g


def fake_quant_fp4(x: Tensor, block_size: int) -> Tensor:
    """MX FP4 QAT quantiser of the last axis: the native kernel on CUDA (block 32, fp32 /
    bf16), the PyTorch statement (``ops.quant.fake_quant_fp4_mx``) otherwise."""
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.quant import fake_quant_fp4_mx

    if (backend.native_for(x) and block_size == 32 and x.shape[-1] % 32 == 0
            and x.dtype in (torch.float32, torch.bfloat16)):
        return _FakeQuantFp4Fn.apply(x)
    return fake_quant_fp4_mx(x, block_size=block_size, axis=-1)


__all__ = ["accumulate_weight_grad", "fake_quant_fp4", "fp8_linear", "fp8_shape_ok", "linear"]

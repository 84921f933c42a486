"""Linear layers and the linear-quantisation factory.

The factory contract matches the reference (``core/quant.py:29-66``):
``factory(in_features, out_features, bias=...) -> nn.Module`` with ``.weight`` /
``.bias`` parameters, so the checkpoint keys are identical under every
``linear_quant`` mode.

* ``Linear`` subclasses ``nn.Linear`` (the reference's ``normal`` init touches
  every ``nn.Linear`` instance, so this keeps init parity) and on CUDA runs our
  sm_100a GEMM.
* ``Fp8Linear`` / ``Fp4Linear`` are *not* ``nn.Linear`` subclasses and keep
  kaiming-uniform init, as in the reference (``kernels/linear_fp8.py:88-93``).
  Eager forward = fake-quant + linear with STE (reference semantics).  On CUDA
  with ``use_real_fp8_gemm`` the forward is this framework's block-scaled FP8
  tensor-core GEMM (1x128 activation / 128x128 weight blocks, UE8M0 scales), a
  finer-grained recipe than the reference's row/column ``_scaled_mm``.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import Any, Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.ops import backend
from saint_llm_b200.ops.quant import Fp8Format, fake_quant_fp4_mx, fake_quant_fp8

LinearFactory = Callable[..., nn.Module]
LinearQuantMode = Literal["bf16", "fp8", "fp4"]


class Linear(nn.Linear):
    """``nn.Linear`` whose CUDA forward/backward run on the native GEMM."""

    def forward(self, x: Tensor) -> Tensor:
        if backend.native_for(x):
            from saint_llm_b200.ops import linear as lin

            return lin.linear(x, self.weight, self.bias)
        return F.linear(x, self.weight, self.bias)


def default_linear(in_features: int, out_features: int, *, bias: bool = True) -> nn.Module:
    return Linear(in_features, out_features, bias=bias)


# reference-compatible alias
_default_linear = default_linear


class _QuantLinearBase(nn.Module):
    weight: Tensor
    bias: Tensor | None

    def __init__(self, in_features: int, out_features: int, bias: bool = True, *,
                 device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        kw: dict[str, Any] = {}
        if device is not None:
            kw["device"] = device
        if dtype is not None:
            kw["dtype"] = dtype
        self.weight = nn.Parameter(torch.empty((out_features, in_features), **kw))
        if bias:
            self.bias = nn.Parameter(torch.empty((out_features,), **kw))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1.0 / math.sqrt(self.in_features) if self.in_features > 0 else 0.0
            nn.init.uniform_(self.bias, -bound, bound)

    @classmethod
    def _copy_from(cls, layer: _QuantLinearBase, linear: nn.Linear) -> None:
        with torch.no_grad():
            layer.weight.copy_(linear.weight)
            if linear.bias is not None and layer.bias is not None:
                layer.bias.copy_(linear.bias)


class Fp8Linear(_QuantLinearBase):
    """FP8 QAT linear.  Eager: fake-quant (weight per-out-channel, activation per-tensor)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, *,
                 weight_fmt: Fp8Format = Fp8Format.E4M3, activation_fmt: Fp8Format = Fp8Format.E4M3,
                 weight_axis: int | None = 0, activation_axis: int | None = None,
                 use_real_fp8_gemm: bool = False, device: torch.device | None = None,
                 dtype: torch.dtype | None = None) -> None:
        self.weight_fmt = weight_fmt
        self.activation_fmt = activation_fmt
        self.weight_axis = weight_axis
        self.activation_axis = activation_axis
        self.use_real_fp8_gemm = use_real_fp8_gemm
        super().__init__(in_features, out_features, bias, device=device, dtype=dtype)

    def forward(self, x: Tensor) -> Tensor:
        if backend.native_for(x):
            from saint_llm_b200.ops import linear as lin

            if self.use_real_fp8_gemm and lin.fp8_shape_ok(self.in_features, self.out_features):
                return lin.fp8_linear(x, self.weight, self.bias)
        xq = fake_quant_fp8(x, fmt=self.activation_fmt, axis=self.activation_axis)
        wq = fake_quant_fp8(self.weight, fmt=self.weight_fmt, axis=self.weight_axis)
        if backend.native_for(x):
            from saint_llm_b200.ops import linear as lin

            return lin.linear(xq, wq, self.bias)
        return F.linear(xq, wq, self.bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, **kw: Any) -> Fp8Linear:
        layer = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                    device=linear.weight.device, dtype=linear.weight.dtype, **kw)
        cls._copy_from(layer, linear)
        return layer

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, weight_fmt={self.weight_fmt.value}, "
                f"activation_fmt={self.activation_fmt.value}")


class Fp4Linear(_QuantLinearBase):
    """MXFP4 QAT linear: block-``block_size`` fake quant of weight and activation along K."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, *,
                 block_size: int = 32, device: torch.device | None = None,
                 dtype: torch.dtype | None = None) -> None:
        if in_features % block_size:
            raise ValueError(f"in_features={in_features} must be a multiple of block_size={block_size}")
        self.block_size = block_size
        super().__init__(in_features, out_features, bias, device=device, dtype=dtype)

    def forward(self, x: Tensor) -> Tensor:
        if backend.native_for(x):
            from saint_llm_b200.ops import linear as lin

            xq = lin.fake_quant_fp4(x, self.block_size)
            wq = lin.fake_quant_fp4(self.weight, self.block_size)
            return lin.linear(xq, wq, self.bias)
        xq = fake_quant_fp4_mx(x, block_size=self.block_size, axis=-1)
        wq = fake_quant_fp4_mx(self.weight, block_size=self.block_size, axis=-1)
        return F.linear(xq, wq, self.bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, *, block_size: int = 32) -> Fp4Linear:
        layer = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                    block_size=block_size, device=linear.weight.device, dtype=linear.weight.dtype)
        cls._copy_from(layer, linear)
        return layer

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, block_size={self.block_size}")


def make_linear_factory(mode: LinearQuantMode, *, fp4_block_size: int = 32,
                        fp8_use_real_gemm: bool = False) -> LinearFactory:
    if mode == "bf16":
        return default_linear
    if mode == "fp8":
        def fp8_factory(in_features: int, out_features: int, *, bias: bool = True) -> nn.Module:
            return Fp8Linear(in_features, out_features, bias=bias, use_real_fp8_gemm=fp8_use_real_gemm)

        return fp8_factory
    if mode == "fp4":
        def fp4_factory(in_features: int, out_features: int, *, bias: bool = True) -> nn.Module:
            return Fp4Linear(in_features, out_features, bias=bias, block_size=fp4_block_size)

        return fp4_factory
    raise ValueError(f"unknown linear_quant mode: {mode!r}")


__all__ = ["Fp4Linear", "Fp8Linear", "Linear", "LinearFactory", "default_linear", "make_linear_factory"]

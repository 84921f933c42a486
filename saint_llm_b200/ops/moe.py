"""MoE expert pool and the fused MoE layer path.

``GroupedSwiGLUExperts`` keeps the reference's stacked layout
(``kernels/moe_grouped.py:82-214``): ``gate_weight``/``up_weight`` (E, I, D) and
``down_weight`` (E, D, I), each expert initialised kaiming-uniform like an
``nn.Linear`` weight.  Eager forward = expand top-k, stable sort by expert, three
per-expert matmuls with the V4 clamps, gate weighting, ``index_add_``.

``moe_forward`` (CUDA) is the fused layer used by ``DeepSeekMoE`` on the GPU; it is
defined in ``ops.moe_native`` and imported lazily so that CPU-only installs never
touch the extension.
"""

from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.ops.quant import Fp8Format, fake_quant_fp8

GroupedQuantMode = Literal["bf16", "fp8", "fp4"]


def grouped_mm_reference(a: Tensor, b: Tensor, offsets: Tensor) -> Tensor:
    """a (M, K) rows grouped by ``offsets`` (cumulative ends); b (E, K, N) -> (M, N)."""
    out = a.new_zeros(a.shape[0], b.shape[2])
    start = 0
    for e, end in enumerate(offsets.tolist()):
        if end > start:
            out[start:end] = a[start:end] @ b[e]
        start = end
    return out


def grouped_mm(a: Tensor, b: Tensor, offsets: Tensor) -> Tensor:
    if a.is_cuda:
        from saint_llm_b200.ops import backend

        if backend.native_for(a):
            from saint_llm_b200.ops import gemm

            return gemm.grouped_mm(a, b, offsets)
    return grouped_mm_reference(a, b, offsets)


class GroupedSwiGLUExperts(nn.Module):
    def __init__(self, hidden_dim: int, intermediate_dim: int, n_experts: int, *,
                 clamp_linear: tuple[float, float] = (-10.0, 10.0), clamp_gate_max: float = 10.0,
                 linear_quant: GroupedQuantMode = "bf16", fp4_block_size: int = 32,
                 device: torch.device | None = None, dtype: torch.dtype | None = None) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.n_experts = n_experts
        self.clamp_linear = clamp_linear
        self.clamp_gate_max = clamp_gate_max
        self.linear_quant = linear_quant
        self.fp4_block_size = fp4_block_size
        kw = {k: v for k, v in (("device", device), ("dtype", dtype)) if v is not None}
        self.gate_weight = nn.Parameter(torch.empty((n_experts, intermediate_dim, hidden_dim), **kw))
        self.up_weight = nn.Parameter(torch.empty((n_experts, intermediate_dim, hidden_dim), **kw))
        self.down_weight = nn.Parameter(torch.empty((n_experts, hidden_dim, intermediate_dim), **kw))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for w in (self.gate_weight, self.up_weight, self.down_weight):
            for e in range(self.n_experts):
                nn.init.kaiming_uniform_(w[e], a=math.sqrt(5.0))

    def _q_act(self, x: Tensor) -> Tensor:
        if self.linear_quant == "fp8":
            return fake_quant_fp8(x, fmt=Fp8Format.E4M3, axis=0)
        if self.linear_quant == "fp4":
            from saint_llm_b200.ops.linear import fake_quant_fp4

            return fake_quant_fp4(x, self.fp4_block_size)  # native kernel on CUDA
        return x

    def _q_weight(self, w: Tensor) -> Tensor:
        if self.linear_quant == "bf16":
            return w
        flat = w.reshape(w.shape[0] * w.shape[1], -1)
        if self.linear_quant == "fp8":
            q = fake_quant_fp8(flat, fmt=Fp8Format.E4M3, axis=0)
        else:
            from saint_llm_b200.ops.linear import fake_quant_fp4

            q = fake_quant_fp4(flat, self.fp4_block_size)  # native kernel on CUDA
        return q.reshape(w.shape)

    def forward(self, flat_h: Tensor, flat_idx: Tensor, flat_gate: Tensor) -> Tensor:
        m, k = flat_idx.shape
        expert = flat_idx.reshape(-1)
        order = torch.argsort(expert, stable=True)
        token_of = torch.arange(m, device=flat_h.device).repeat_interleave(k)[order]
        x = self._q_act(flat_h.repeat_interleave(k, dim=0)[order])
        offsets = torch.cumsum(torch.bincount(expert, minlength=self.n_experts), 0).to(torch.int32)
        wg = self._q_weight(self.gate_weight).transpose(1, 2)
        wu = self._q_weight(self.up_weight).transpose(1, 2)
        wd = self._q_weight(self.down_weight).transpose(1, 2)
        g = grouped_mm(x, wg, offsets).clamp(max=self.clamp_gate_max)
        u = grouped_mm(x, wu, offsets).clamp(min=self.clamp_linear[0], max=self.clamp_linear[1])
        y = grouped_mm(self._q_act(F.silu(g) * u), wd, offsets)
        y = y * flat_gate.reshape(-1)[order].unsqueeze(-1).to(y.dtype)
        return flat_h.new_zeros(m, self.hidden_dim).index_add_(0, token_of, y.to(flat_h.dtype))


def moe_forward(layer: nn.Module, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
    from saint_llm_b200.ops import moe_native

    return moe_native.moe_forward(layer, x, token_ids, is_visual)


__all__ = ["GroupedSwiGLUExperts", "grouped_mm", "grouped_mm_reference", "moe_forward"]

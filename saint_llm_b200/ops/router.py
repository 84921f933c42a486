"""Fused MoE router (``csrc/router.cu``): one forward kernel and one backward kernel.

The forward computes the affinity (``sqrt(softplus(z))`` or ``sigmoid(z)``), the
bias-adjusted top-k selection and the renormalised gates.  The backward (one warp per
token) folds the gates' renormalisation, the affinity gradient coming from the
sequence-balance loss and the affinity's derivative into dz.  The biases only steer the
selection, so they get no gradient (as with ``topk`` indices in the eager router).
"""

from __future__ import annotations

import torch
from torch import Tensor

from saint_llm_b200.ops import backend


class _RouteFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z: Tensor, k: int, mode: int, bias: Tensor | None, mbias: Tensor | None,  # type: ignore[override]
                visual: Tensor | None):
        lead, e = z.shape[:-1], z.shape[-1]
        z2 = z.reshape(-1, e).float().contiguous()
        t = z2.shape[0]
        aff = torch.empty_like(z2)
        idx = torch.empty(t, k, dtype=torch.int64, device=z.device)
        gate = torch.empty(t, k, dtype=torch.float32, device=z.device)
        backend.ext().router_fwd(z2, k, mode, None if bias is None else bias.float().contiguous(),
                                 None if mbias is None else mbias.float().contiguous(),
                                 None if visual is None else visual.reshape(-1).bool().contiguous(), aff, idx, gate)
        ctx.save_for_backward(z2, aff, idx, gate)
        ctx.mode, ctx.lead = mode, lead
        ctx.mark_non_differentiable(idx)
        return idx.view(*lead, k), gate.view(*lead, k), aff.view(*lead, e)

    @staticmethod
    def backward(ctx, d_idx, d_gate: Tensor | None, d_aff: Tensor | None):  # type: ignore[override]
        z2, aff, idx, gate = ctx.saved_tensors
        e = aff.shape[-1]
        dz = torch.empty_like(z2)
        dg = None if d_gate is None else d_gate.reshape(-1, gate.shape[-1]).float().contiguous()
        da = None if d_aff is None else d_aff.reshape(-1, e).float().contiguous()
        backend.ext().router_bwd(z2, aff, idx, gate, dg, da, ctx.mode, dz)
        return dz.view(*ctx.lead, e), None, None, None, None, None


def route_backward_reference(z: Tensor, aff: Tensor, idx: Tensor, gate: Tensor, d_gate: Tensor | None,
                             d_aff: Tensor | None, mode: int) -> Tensor:
    """PyTorch statement of the backward kernel (its test oracle)."""
    da = torch.zeros_like(aff) if d_aff is None else d_aff.float().clone()
    if d_gate is not None:
        s = aff.gather(-1, idx).sum(-1, keepdim=True) + 1.0e-12
        d_raw = (d_gate - (d_gate * gate).sum(-1, keepdim=True)) / s
        da.scatter_add_(-1, idx, d_raw)
    if mode == 0:   # aff = sqrt(softplus(z) + eps): d aff / dz = sigmoid(z) / (2 aff)
        return da * torch.sigmoid(z) / (2.0 * aff)
    return da * aff * (1.0 - aff)


def fused_route(logits: Tensor, k: int, affinity_fn: str, bias: Tensor | None, modality_bias: Tensor | None,
                is_visual: Tensor | None) -> tuple[Tensor, Tensor, Tensor]:
    """(expert_idx, renormalised gates, affinity) of the learned router, as ``LearnedRouter``."""
    mode = 0 if affinity_fn == "sqrt_softplus" else 1
    vis = is_visual if modality_bias is not None else None
    return _RouteFn.apply(logits, k, mode, bias, modality_bias if vis is not None else None, vis)


__all__ = ["fused_route", "route_backward_reference"]

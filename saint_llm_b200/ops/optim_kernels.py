"""Optimizer update sweeps for the CUDA path.

``adamw_step`` applies decoupled-weight-decay Adam to a list of parameters with fp32
state, reading the fp32 ``main_grad`` when present, as one multi-tensor sweep per
state tensor.
"""

from __future__ import annotations

import torch
from torch import Tensor


def _grad(p: Tensor) -> Tensor:
    mg = getattr(p, "main_grad", None)
    return mg if mg is not None else p.grad


@torch.no_grad()
def adamw_step(params: list[Tensor], states: list[dict], *, lr: float, beta1: float, beta2: float, eps: float,
               weight_decay: float) -> None:
    grads = [_grad(p).float() for p in params]
    m = [s["exp_avg"] for s in states]
    v = [s["exp_avg_sq"] for s in states]
    for s in states:
        s["step"] += 1
    t = float(states[0]["step"])
    torch._foreach_mul_(m, beta1)
    torch._foreach_add_(m, grads, alpha=1 - beta1)
    torch._foreach_mul_(v, beta2)
    torch._foreach_addcmul_(v, grads, grads, value=1 - beta2)
    bc1, bc2 = 1 - beta1 ** t, 1 - beta2 ** t
    denom = torch._foreach_div(v, bc2)
    torch._foreach_sqrt_(denom)
    torch._foreach_add_(denom, eps)
    upd = torch._foreach_div(m, denom)
    torch._foreach_mul_(upd, 1.0 / bc1)
    for p, u in zip(params, upd, strict=True):
        p.mul_(1 - lr * weight_decay).add_(u.to(p.dtype), alpha=-lr)

"""Optimizer update sweeps for the CUDA path.

``adamw_step`` applies decoupled-weight-decay Adam to a list of parameters with fp32
state, reading the fp32 ``main_grad`` when present, in ONE native launch
(``csrc/optim.cu: adamw_multi``): a device table of (gradient, parameter, moments, size,
dtype) rows and a chunk list built once per parameter set and reused every step (the
pointers never move).  The step count lives on the host next to the table, so computing
the bias corrections needs no device read; the state's ``step`` tensor is still advanced
on the device for checkpoints.
"""

from __future__ import annotations

import torch
from torch import Tensor

_TABLES: dict[tuple, tuple[Tensor, Tensor, list]] = {}


def _grad(p: Tensor) -> Tensor:
    mg = getattr(p, "main_grad", None)
    return mg if mg is not None else p.grad


def _table(params: list[Tensor], states: list[dict]) -> tuple[Tensor, Tensor, list]:
    from saint_llm_b200.ops import backend

    grads = [_grad(p) for p in params]
    key = tuple((p.data_ptr(), g.data_ptr(), s["exp_avg"].data_ptr(), s["exp_avg_sq"].data_ptr())
                for p, g, s in zip(params, grads, states, strict=True))
    hit = _TABLES.get(key)
    if hit is not None:
        return hit
    ext = backend.ext()
    chunk = ext.adamw_chunk_elems()
    rows, chunks, keep = [], [], []
    for i, (p, g, s) in enumerate(zip(params, grads, states, strict=True)):
        if g.dtype != torch.float32 or not g.is_contiguous() or not p.is_contiguous() or p.dtype not in (
                torch.bfloat16, torch.float32):
            raise ValueError("adamw_step needs contiguous fp32 gradients and bf16 / fp32 parameters")
        keep.append((p, g, s))
        rows.append([g.data_ptr(), p.data_ptr(), s["exp_avg"].data_ptr(), s["exp_avg_sq"].data_ptr(), p.numel(),
                     int(p.dtype == torch.bfloat16)])
        chunks += [(i << 32) | c for c in range((p.numel() + chunk - 1) // chunk)]
    dev = params[0].device
    table = torch.tensor(rows, dtype=torch.int64).to(dev)
    chunk_t = torch.tensor(chunks, dtype=torch.int64).to(dev)
    _TABLES[key] = (table, chunk_t, keep)
    return _TABLES[key]


@torch.no_grad()
def adamw_step(params: list[Tensor], states: list[dict], *, lr: float, beta1: float, beta2: float, eps: float,
               weight_decay: float) -> None:
    from saint_llm_b200.ops import backend

    table, chunks, _ = _table(params, states)
    prev = states[0].get("host_step")
    if prev is None:  # fresh state, or one restored from a checkpoint (one read)
        prev = int(states[0]["step"].item())
    host_t = prev + 1
    for s in states:
        s["host_step"] = host_t
        s["step"] += 1
    backend.ext().adamw_multi(table, chunks, lr, beta1, beta2, eps, weight_decay, float(host_t))

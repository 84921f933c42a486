"""On-policy distillation from several teachers (reference: ``saint_llm_posttraining/opd.py``).

Teachers are pooled into one distribution (uniform or weighted mixture in probability
space, or per-position the most confident teacher), and the student minimises the
forward KL(student || teacher) at temperature T, scaled by T^2, over response positions.
The KL is evaluated in row chunks so only a chunk of (rows, V) fp32 intermediates exists
at a time.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn

Aggregation = Literal["mean", "weighted", "max"]


@dataclass(frozen=True)
class OPDConfig:
    temperature: float = 1.0
    aggregation: Aggregation = "mean"
    kl_coef: float = 1.0


def aggregate_teacher_logits(teacher_logits: Sequence[Tensor], *, weights: Tensor | None = None,
                             mode: Aggregation = "mean") -> Tensor:
    """K teachers' (B, T, V) logits -> pooled (B, T, V) log-probabilities."""
    if not teacher_logits:
        raise ValueError("teacher_logits is empty")
    if len({tuple(t.shape) for t in teacher_logits}) != 1 or teacher_logits[0].dim() != 3:
        raise ValueError("teachers must share one (B, T, V) shape")
    stack = torch.stack([t.float() for t in teacher_logits])
    if mode == "max":
        pick = stack.amax(-1).argmax(0)  # (B, T): teacher with the largest top-1 logit
        chosen = stack.gather(0, pick[None, ..., None].expand(1, *stack.shape[1:])).squeeze(0)
        return F.log_softmax(chosen, -1)
    k = stack.shape[0]
    if mode == "mean":
        w = torch.full((k,), 1.0 / k, device=stack.device)
    elif mode == "weighted":
        if weights is None:
            raise ValueError("weighted aggregation requires 'weights'")
        if weights.shape != (k,):
            raise ValueError(f"weights shape {tuple(weights.shape)} must be ({k},)")
        if not torch.isclose(weights.sum().float().cpu(), torch.tensor(1.0)):
            raise ValueError(f"weights must sum to 1; got {float(weights.sum())}")
        w = weights.float().to(stack.device)
    else:
        raise ValueError(f"unknown aggregation mode: {mode!r}")
    return torch.logsumexp(F.log_softmax(stack, -1) + torch.log(w + 1e-12).view(-1, 1, 1, 1), dim=0)


def opd_kl_loss(student_logits: Tensor, teacher_log_probs: Tensor, response_mask: Tensor, *,
                temperature: float = 1.0, chunk_rows: int = 2048) -> tuple[Tensor, int]:
    if student_logits.shape != teacher_log_probs.shape:
        raise ValueError(f"student / teacher shapes differ: {tuple(student_logits.shape)} vs "
                         f"{tuple(teacher_log_probs.shape)}")
    if temperature <= 0.0:
        raise ValueError(f"temperature must be positive; got {temperature}")
    v = student_logits.shape[-1]
    s2, t2 = student_logits.reshape(-1, v), teacher_log_probs.reshape(-1, v)
    mask = response_mask.reshape(-1).to(student_logits.device, torch.float32)
    total = student_logits.new_zeros((), dtype=torch.float32)
    for r0 in range(0, s2.shape[0], chunk_rows):
        sl = F.log_softmax(s2[r0:r0 + chunk_rows].float() / temperature, -1)
        tl = F.log_softmax(t2[r0:r0 + chunk_rows].float() / temperature, -1)
        kl = (sl.exp() * (sl - tl)).sum(-1)
        total = total + (kl * mask[r0:r0 + chunk_rows]).sum()
    n = int(mask.sum())
    return total / mask.sum().clamp(min=1.0) * temperature ** 2, n


def opd_step(student: nn.Module, teachers: Sequence[nn.Module], tokens: Tensor, response_mask: Tensor, *,
             cfg: OPDConfig, teacher_weights: Tensor | None = None) -> tuple[Tensor, dict[str, Tensor]]:
    s_logits = student(tokens)["logits"]
    with torch.no_grad():
        pooled = aggregate_teacher_logits([t(tokens)["logits"] for t in teachers], weights=teacher_weights,
                                          mode=cfg.aggregation)
    kl, n = opd_kl_loss(s_logits, pooled, response_mask, temperature=cfg.temperature)
    loss = cfg.kl_coef * kl
    dev = loss.device
    return loss, {"kl": kl.detach(), "n_active": torch.tensor(n, device=dev),
                  "n_teachers": torch.tensor(len(teachers), device=dev)}


__all__ = ["OPDConfig", "aggregate_teacher_logits", "opd_kl_loss", "opd_step"]

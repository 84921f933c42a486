"""Process reward model over reasoning steps: a small MLP scores the hidden state at each
step-boundary token (reference: ``saint_llm_posttraining/think_prm.py:48-235``).  Step
positions are found for the whole batch at once (no per-row Python loop)."""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn


@dataclass(frozen=True)
class ThinkPRMConfig:
    hidden_dim: int
    intermediate: int = 0  # 0 -> 2 * hidden_dim
    threshold: float = 0.5
    keep_min_step_score: float = 0.4

    def effective_intermediate(self) -> int:
        return self.intermediate if self.intermediate > 0 else 2 * self.hidden_dim


class StepRewardHead(nn.Module):
    def __init__(self, cfg: ThinkPRMConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.fc1 = nn.Linear(cfg.hidden_dim, cfg.effective_intermediate())
        self.fc2 = nn.Linear(cfg.effective_intermediate(), 1)

    def forward(self, hidden: Tensor) -> Tensor:
        return self.fc2(F.gelu(self.fc1(hidden)))


def find_step_boundaries(tokens: Tensor, boundary_id: int) -> Tensor:
    """(B, T) -> (B, T): each row's boundary positions in order, then -1 padding."""
    if tokens.dim() != 2:
        raise ValueError(f"tokens must be (B, T); got {tuple(tokens.shape)}")
    b, t = tokens.shape
    hit = tokens == boundary_id
    slot = hit.long().cumsum(1) - 1  # rank of each boundary within its row
    out = torch.full((b, t), -1, dtype=torch.long, device=tokens.device)
    rows, cols = hit.nonzero(as_tuple=True)
    out[rows, slot[rows, cols]] = cols
    return out


def gather_step_logits(hidden: Tensor, head: StepRewardHead, step_positions: Tensor) -> tuple[Tensor, Tensor]:
    if hidden.dim() != 3:
        raise ValueError(f"hidden must be (B, T, D); got {tuple(hidden.shape)}")
    if step_positions.shape[0] != hidden.shape[0]:
        raise ValueError("step_positions batch size differs from hidden")
    valid = step_positions >= 0
    g = hidden.gather(1, step_positions.clamp(min=0).unsqueeze(-1).expand(-1, -1, hidden.shape[-1]))
    return head(g).squeeze(-1).masked_fill(~valid, 0.0), valid


def gather_step_scores(hidden: Tensor, head: StepRewardHead, step_positions: Tensor) -> tuple[Tensor, Tensor]:
    logits, valid = gather_step_logits(hidden, head, step_positions)
    return torch.sigmoid(logits).masked_fill(~valid, 0.0), valid


def step_prm_loss(logits: Tensor, labels: Tensor, mask: Tensor, *, pos_weight: float | None = None) -> Tensor:
    if logits.shape != labels.shape or logits.shape != mask.shape:
        raise ValueError("logits, labels, mask must share shape")
    pw = torch.tensor(pos_weight, device=logits.device, dtype=logits.dtype) if pos_weight is not None else None
    el = F.binary_cross_entropy_with_logits(logits, labels.float(), reduction="none", pos_weight=pw) * mask.float()
    return el.sum() / mask.float().sum().clamp(min=1.0)


def compute_step_rewards(hidden: Tensor, head: StepRewardHead, tokens: Tensor, boundary_id: int
                         ) -> tuple[Tensor, Tensor]:
    return gather_step_scores(hidden, head, find_step_boundaries(tokens, boundary_id))


def prm_filter_mask(probs: Tensor, valid: Tensor, *, min_score: float) -> Tensor:
    """Keep a trace iff every real step scores >= min_score (rows without steps are kept)."""
    if probs.shape != valid.shape:
        raise ValueError("probs and valid must share shape")
    return ~((probs < min_score) & valid).any(-1)


__all__ = ["StepRewardHead", "ThinkPRMConfig", "compute_step_rewards", "find_step_boundaries", "gather_step_logits",
           "gather_step_scores", "prm_filter_mask", "step_prm_loss"]

"""GTPO: GRPO with per-token advantages weighted by the policy's entropy at that token
(reference: ``saint_llm_posttraining/gtpo.py:62-248``).  weight = (1 - alpha) + alpha * H_t /
max response H (per row, or the batch max)."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch.nn.functional as F
from torch import Tensor

from saint_llm_b200.posttrain.grpo import (
    GRPOConfig,
    RolloutBatch,
    compute_group_advantage,
    gather_token_logprobs,
    policy_surrogate_loss,
)


@dataclass(frozen=True)
class GTPOConfig:
    grpo: GRPOConfig = field(default_factory=GRPOConfig)
    entropy_alpha: float = 0.5
    normalize_per_row: bool = True

    def __post_init__(self) -> None:
        if not 0.0 <= self.entropy_alpha <= 1.0:
            raise ValueError(f"entropy_alpha must be in [0, 1]; got {self.entropy_alpha}")


def per_token_entropy(logits: Tensor) -> Tensor:
    if logits.dim() != 3:
        raise ValueError(f"logits must be (B, T, V); got shape {tuple(logits.shape)}")
    lp = F.log_softmax(logits.detach().float(), -1)
    return -(lp.exp() * lp).sum(-1)


def entropy_weight(entropy: Tensor, response_mask: Tensor, *, alpha: float, normalize_per_row: bool = True,
                   eps: float = 1e-8) -> Tensor:
    if entropy.shape != response_mask.shape:
        raise ValueError(f"entropy {tuple(entropy.shape)} and mask {tuple(response_mask.shape)} differ")
    if not 0.0 <= alpha <= 1.0:
        raise ValueError(f"alpha must be in [0, 1]; got {alpha}")
    mask = response_mask.to(entropy.dtype)
    h = entropy * mask
    denom = (h.amax(-1, keepdim=True) if normalize_per_row else h.max()).clamp(min=eps)
    return ((1.0 - alpha) + alpha * (h / denom).clamp(0.0, 1.0)) * mask


def gtpo_loss(logits: Tensor, batch: RolloutBatch, *, cfg: GTPOConfig) -> tuple[Tensor, dict[str, Tensor]]:
    g = cfg.grpo
    new = gather_token_logprobs(logits, batch.tokens)
    adv = compute_group_advantage(batch.rewards, group_size=g.group_size, eps=g.advantage_eps,
                                  unbiased=g.unbiased_loss)
    ent = per_token_entropy(logits)
    w = entropy_weight(ent, batch.response_mask, alpha=cfg.entropy_alpha, normalize_per_row=cfg.normalize_per_row)
    loss, m = policy_surrogate_loss(new, batch, adv, g, token_weight=w.to(new.dtype))
    mask = batch.response_mask.to(ent.dtype)
    denom = mask.sum().clamp(min=1.0)
    m["mean_entropy_weight"] = ((w * mask).sum() / denom).detach()
    m["mean_entropy_nats"] = ((ent * mask).sum() / denom).detach()
    return loss, m


__all__ = ["GTPOConfig", "entropy_weight", "gtpo_loss", "per_token_entropy"]

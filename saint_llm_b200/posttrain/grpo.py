"""GRPO-family policy-gradient math.

Reference behaviour (``saint_llm_posttraining/grpo.py:43-340``): group-normalised
advantages (Dr.GRPO drops the std), DAPO dynamic sampling and overlong reward shaping,
the PPO clipped surrogate with symmetric or Clip-Higher bounds, a token- or
sequence-level (GSPO) importance ratio, the k3 estimator of KL to the reference policy,
and mean-over-tokens vs token-level (DAPO) aggregation.

Here all variants (GRPO, GTPO's entropy-weighted tokens, Tree-GRPO's sibling groups)
share one surrogate, :func:`policy_surrogate_loss`, fed with per-token log-probabilities.
On CUDA those come from :func:`policy_token_logprobs`, which runs the backbone and the
fused LM-head log-prob kernel: the (rows, vocab) logits are never materialised, in the
forward or the backward.  ``grpo_loss(logits, ...)`` keeps the logits-based signature.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor, nn


@dataclass(frozen=True)
class GRPOConfig:
    group_size: int = 8
    clip_eps: float = 0.2
    clip_eps_upper: float = 0.28
    clip_eps_lower: float = 0.20
    use_clip_higher: bool = False
    kl_coef: float = 0.04
    advantage_eps: float = 1e-8
    importance_ratio_level: Literal["token", "sequence"] = "token"
    token_level_pg: bool = False
    overlong_reward_band: tuple[float, float] | None = None
    unbiased_loss: bool = False

    @property
    def clip_bounds(self) -> tuple[float, float]:
        if self.use_clip_higher:
            return 1.0 - self.clip_eps_lower, 1.0 + self.clip_eps_upper
        return 1.0 - self.clip_eps, 1.0 + self.clip_eps


@dataclass(frozen=True)
class RolloutBatch:
    """Rows ``[b*G, (b+1)*G)`` are the G completions of prompt b.  Log-prob tensors are
    aligned with ``tokens``: entry t is log pi(tokens[t] | tokens[<t]), entry 0 is 0."""

    tokens: Tensor
    response_mask: Tensor
    old_logprobs: Tensor
    ref_logprobs: Tensor
    rewards: Tensor

    def select(self, idx: Tensor) -> RolloutBatch:
        return RolloutBatch(self.tokens[idx], self.response_mask[idx], self.old_logprobs[idx],
                            self.ref_logprobs[idx], self.rewards[idx])


def _groups(rewards: Tensor, group_size: int) -> Tensor:
    if group_size <= 0:
        raise ValueError(f"group_size must be positive; got {group_size}")
    if rewards.shape[0] % group_size:
        raise ValueError(f"rewards length {rewards.shape[0]} is not divisible by group_size {group_size}")
    return rewards.view(-1, group_size)


def compute_group_advantage(rewards: Tensor, *, group_size: int, eps: float = 1e-8, unbiased: bool = False) -> Tensor:
    g = _groups(rewards, group_size)
    centred = g - g.mean(-1, keepdim=True)
    return (centred if unbiased else centred / (g.std(-1, unbiased=False, keepdim=True) + eps)).reshape(-1)


def dynamic_sampling_mask(rewards: Tensor, *, group_size: int) -> Tensor:
    """True for rows of groups whose rewards are not all equal (DAPO dynamic sampling)."""
    g = _groups(rewards, group_size)
    return (g.var(-1, unbiased=False) > 0).repeat_interleave(group_size)


def overlong_reward_shape(rewards: Tensor, response_lengths: Tensor, *, max_length: int,
                          band: tuple[float, float] | None) -> Tensor:
    """Linear decay of the reward from 1x at ``a * max_length`` to 0x at ``b * max_length``."""
    if band is None:
        return rewards
    a, b = band
    if not 0.0 < a < b <= 1.0:
        raise ValueError(f"band must satisfy 0 < a < b <= 1; got {band}")
    frac = response_lengths.to(rewards.dtype) / max(max_length, 1)
    return rewards * ((b - frac) / (b - a)).clamp(0.0, 1.0)


def gather_token_logprobs(logits: Tensor, tokens: Tensor) -> Tensor:
    """(B, T, V) logits -> (B, T): entry t = log p(tokens[t] | < t), entry 0 = 0."""
    if logits.dim() != 3:
        raise ValueError(f"logits must be (B, T, V); got shape {tuple(logits.shape)}")
    if tokens.shape != logits.shape[:2]:
        raise ValueError(f"tokens shape {tuple(tokens.shape)} must match logits[:, :, 0] {tuple(logits.shape[:2])}")
    lp = F.log_softmax(logits[:, :-1].float(), dim=-1).gather(-1, tokens[:, 1:, None]).squeeze(-1)
    return F.pad(lp, (1, 0))


def policy_token_logprobs(model: nn.Module, tokens: Tensor, *, vision_features: Tensor | None = None,
                          audio_features: Tensor | None = None) -> Tensor:
    """(B, T) per-token log-probs of ``tokens`` under ``model`` (entry 0 = 0), differentiable.

    On CUDA: backbone + the fused LM-head log-prob kernel (no logits tensor).  Elsewhere:
    the model's logits and a log-softmax gather."""
    from saint_llm_b200.ops import backend

    if hasattr(model, "backbone") and backend.native_for(next(model.parameters())):
        from saint_llm_b200.ops.ce import token_logprobs

        h, _ = model.backbone(tokens, vision_features, audio_features)
        lp = token_logprobs(h[:, :-1], model.lm_head.weight, tokens[:, 1:],
                            softcap=model.cfg.final_logit_softcap)
        return F.pad(lp, (1, 0))
    kw = {k: v for k, v in (("vision_features", vision_features), ("audio_features", audio_features))
          if v is not None}
    return gather_token_logprobs(model(tokens, **kw)["logits"], tokens)


def policy_surrogate_loss(new_logprobs: Tensor, batch: RolloutBatch, advantages: Tensor, cfg: GRPOConfig, *,
                          token_weight: Tensor | None = None) -> tuple[Tensor, dict[str, Tensor]]:
    """Clipped surrogate + k3 KL over the response tokens; ``token_weight`` (B, T) scales the
    per-token advantage (GTPO)."""
    mask = batch.response_mask.to(new_logprobs.dtype)
    n_tok = mask.sum(-1).clamp(min=1.0)
    log_ratio = new_logprobs - batch.old_logprobs.to(new_logprobs.dtype)
    if cfg.importance_ratio_level == "sequence":
        ratio = ((log_ratio * mask).sum(-1) / n_tok).exp().unsqueeze(-1).expand_as(log_ratio)
    else:
        ratio = log_ratio.exp()
    adv = advantages.to(new_logprobs.dtype).unsqueeze(-1)
    if token_weight is not None:
        adv = adv * token_weight
    lo, hi = cfg.clip_bounds
    s1, s2 = ratio * adv, ratio.clamp(lo, hi) * adv
    objective = torch.minimum(s1, s2)
    kl_log = batch.ref_logprobs.to(new_logprobs.dtype) - new_logprobs
    kl_tok = kl_log.exp() - kl_log - 1.0
    pg = -(objective * mask).sum(-1)
    kl = (kl_tok * mask).sum(-1)
    if not (cfg.token_level_pg or cfg.unbiased_loss):
        pg, kl = pg / n_tok, kl / n_tok
    loss = (pg + cfg.kl_coef * kl).mean()
    with torch.no_grad():
        denom = mask.sum().clamp(min=1.0)
        metrics = {
            "pg_loss": pg.mean(), "kl_penalty": kl.mean(),
            "clip_frac": ((s1 != s2).to(mask.dtype) * mask).sum() / denom,
            "advantage_mean": advantages.mean(), "advantage_std": advantages.std(unbiased=False),
            "reward_mean": batch.rewards.mean(), "ratio_mean": (ratio * mask).sum() / denom,
        }
    return loss, metrics


def grpo_loss_from_logprobs(new_logprobs: Tensor, batch: RolloutBatch, *, cfg: GRPOConfig
                            ) -> tuple[Tensor, dict[str, Tensor]]:
    adv = compute_group_advantage(batch.rewards, group_size=cfg.group_size, eps=cfg.advantage_eps,
                                  unbiased=cfg.unbiased_loss)
    return policy_surrogate_loss(new_logprobs, batch, adv, cfg)


def grpo_loss(logits: Tensor, batch: RolloutBatch, *, cfg: GRPOConfig) -> tuple[Tensor, dict[str, Tensor]]:
    return grpo_loss_from_logprobs(gather_token_logprobs(logits, batch.tokens), batch, cfg=cfg)


__all__ = ["GRPOConfig", "RolloutBatch", "compute_group_advantage", "dynamic_sampling_mask", "gather_token_logprobs",
           "grpo_loss", "grpo_loss_from_logprobs", "overlong_reward_shape", "policy_surrogate_loss",
           "policy_token_logprobs"]

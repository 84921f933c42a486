"""GRPO driver: old/reference log-probs, dynamic-sampling filter, one update
(reference: ``saint_llm_posttraining/grpo_trainer.py:42-186``).  Log-probs come from
:func:`policy_token_logprobs` (fused LM-head kernel on CUDA)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch
from torch import Tensor, nn

from saint_llm_b200.posttrain.grpo import (
    GRPOConfig,
    RolloutBatch,
    dynamic_sampling_mask,
    grpo_loss_from_logprobs,
    policy_token_logprobs,
)


class RewardFn(Protocol):
    def __call__(self, prompt: str, completion: str) -> float: ...


@dataclass
class GRPOTrainerStep:
    loss: Tensor
    metrics: dict[str, Tensor]
    n_kept_groups: int


@torch.no_grad()
def frozen_logprobs(model: nn.Module, tokens: Tensor, **features: Tensor | None) -> Tensor:
    was = model.training
    model.eval()
    try:
        return policy_token_logprobs(model, tokens, **features).detach()
    finally:
        model.train(was)


def build_rollout_batch(*, actor: nn.Module, ref: nn.Module | None, tokens: Tensor, response_mask: Tensor,
                        rewards: Tensor) -> RolloutBatch:
    """``ref=None``: reference log-probs equal the old ones (the KL term is exactly zero)."""
    old = frozen_logprobs(actor, tokens)
    refl = frozen_logprobs(ref, tokens) if ref is not None else old.clone()
    return RolloutBatch(tokens, response_mask, old, refl, rewards)


def _no_signal(batch: RolloutBatch) -> GRPOTrainerStep:
    zero = torch.zeros((), device=batch.rewards.device, requires_grad=True)
    return GRPOTrainerStep(zero, {"reward_mean": batch.rewards.mean().detach()}, 0)


def grpo_train_step(*, actor: nn.Module, optimizer: torch.optim.Optimizer, batch: RolloutBatch,
                    cfg: GRPOConfig) -> GRPOTrainerStep:
    keep = dynamic_sampling_mask(batch.rewards, group_size=cfg.group_size)
    n_groups = int(keep.view(-1, cfg.group_size)[:, 0].sum())
    if n_groups == 0:
        return _no_signal(batch)
    if n_groups * cfg.group_size != keep.numel():
        batch = batch.select(keep.nonzero().squeeze(-1))
    actor.train()
    loss, metrics = grpo_loss_from_logprobs(policy_token_logprobs(actor, batch.tokens), batch, cfg=cfg)
    optimizer.zero_grad(set_to_none=True)
    loss.backward()
    optimizer.step()
    return GRPOTrainerStep(loss.detach(), metrics, n_groups)


def score_rollouts(*, prompts: list[str], completions: list[str], reward_fn: RewardFn) -> Tensor:
    if len(prompts) != len(completions):
        raise ValueError(f"prompts/completions length mismatch: {len(prompts)} vs {len(completions)}")
    return torch.tensor([float(reward_fn(p, c)) for p, c in zip(prompts, completions, strict=True)],
                        dtype=torch.float32)


__all__ = ["GRPOTrainerStep", "RewardFn", "build_rollout_batch", "frozen_logprobs", "grpo_train_step",
           "score_rollouts"]

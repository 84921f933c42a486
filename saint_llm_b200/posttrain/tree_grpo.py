"""Tree-GRPO: advantages normalised within sibling groups of a rollout tree, and its driver
(reference: ``saint_llm_posttraining/tree_grpo.py``, ``tree_grpo_trainer.py``).  Roots form one
group (parent -1); a group with a single member gets advantage 0."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.posttrain.grpo import (
    GRPOConfig,
    RolloutBatch,
    gather_token_logprobs,
    policy_surrogate_loss,
    policy_token_logprobs,
)
from saint_llm_b200.posttrain.trainer import frozen_logprobs


@dataclass(frozen=True)
class TreeRolloutBatch:
    tokens: Tensor
    response_mask: Tensor
    old_logprobs: Tensor
    ref_logprobs: Tensor
    rewards: Tensor
    parent_idx: Tensor

    def flat(self) -> RolloutBatch:
        return RolloutBatch(self.tokens, self.response_mask, self.old_logprobs, self.ref_logprobs, self.rewards)

    def select(self, idx: Tensor) -> TreeRolloutBatch:
        return TreeRolloutBatch(self.tokens[idx], self.response_mask[idx], self.old_logprobs[idx],
                                self.ref_logprobs[idx], self.rewards[idx], self.parent_idx[idx])


def _sibling_stats(rewards: Tensor, parent_idx: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Per-row (group mean, group population variance, group size) via scatter reductions."""
    if rewards.dim() != 1 or rewards.shape != parent_idx.shape:
        raise ValueError(f"rewards {tuple(rewards.shape)} and parent_idx {tuple(parent_idx.shape)} must be 1-D, equal")
    _, gid = torch.unique(parent_idx, return_inverse=True)
    n_g = int(gid.max()) + 1 if gid.numel() else 0
    r = rewards.float()
    cnt = torch.zeros(n_g, device=r.device).index_add_(0, gid, torch.ones_like(r))
    mean = torch.zeros(n_g, device=r.device).index_add_(0, gid, r) / cnt
    var = torch.zeros(n_g, device=r.device).index_add_(0, gid, (r - mean[gid]) ** 2) / cnt
    return mean[gid], var[gid], cnt[gid]


def compute_tree_advantage(rewards: Tensor, parent_idx: Tensor, *, eps: float = 1e-8,
                           unbiased: bool = False) -> Tensor:
    mean, var, cnt = _sibling_stats(rewards, parent_idx)
    adv = rewards.float() - mean
    if not unbiased:
        adv = adv / (var.sqrt() + eps)
    return torch.where(cnt > 1, adv, torch.zeros_like(adv)).to(rewards.dtype)


def tree_dynamic_sampling_mask(rewards: Tensor, parent_idx: Tensor) -> Tensor:
    """Drop sibling groups (size > 1) whose rewards are all equal; singletons are kept."""
    _, var, cnt = _sibling_stats(rewards, parent_idx)
    return (cnt <= 1) | (var > 0)


def tree_grpo_loss_from_logprobs(new_logprobs: Tensor, batch: TreeRolloutBatch, *, cfg: GRPOConfig
                                 ) -> tuple[Tensor, dict[str, Tensor]]:
    adv = compute_tree_advantage(batch.rewards, batch.parent_idx, eps=cfg.advantage_eps, unbiased=cfg.unbiased_loss)
    loss, m = policy_surrogate_loss(new_logprobs, batch.flat(), adv, cfg)
    m["n_sibling_groups"] = torch.tensor(int(torch.unique(batch.parent_idx).numel()), device=loss.device)
    return loss, m


def tree_grpo_loss(logits: Tensor, batch: TreeRolloutBatch, *, cfg: GRPOConfig) -> tuple[Tensor, dict[str, Tensor]]:
    return tree_grpo_loss_from_logprobs(gather_token_logprobs(logits, batch.tokens), batch, cfg=cfg)


@dataclass
class TreeGRPOTrainerStep:
    loss: Tensor
    metrics: dict[str, Tensor]
    n_kept_groups: int


def build_tree_rollout_batch(*, actor: nn.Module, ref: nn.Module | None, tokens: Tensor, response_mask: Tensor,
                             rewards: Tensor, parent_idx: Tensor) -> TreeRolloutBatch:
    old = frozen_logprobs(actor, tokens)
    refl = frozen_logprobs(ref, tokens) if ref is not None else old.clone()
    return TreeRolloutBatch(tokens, response_mask, old, refl, rewards, parent_idx)


def tree_grpo_train_step(*, actor: nn.Module, optimizer: torch.optim.Optimizer, batch: TreeRolloutBatch,
                         cfg: GRPOConfig) -> TreeGRPOTrainerStep:
    keep = tree_dynamic_sampling_mask(batch.rewards, batch.parent_idx)
    if not bool(keep.any()):
        zero = torch.zeros((), device=batch.rewards.device, requires_grad=True)
        return TreeGRPOTrainerStep(zero, {"reward_mean": batch.rewards.mean().detach()}, 0)
    if not bool(keep.all()):
        batch = batch.select(keep.nonzero().squeeze(-1))
    actor.train()
    loss, m = tree_grpo_loss_from_logprobs(policy_token_logprobs(actor, batch.tokens), batch, cfg=cfg)
    optimizer.zero_grad(set_to_none=True)
    loss.backward()
    optimizer.step()
    return TreeGRPOTrainerStep(loss.detach(), m, int(torch.unique(batch.parent_idx).numel()))


__all__ = ["TreeGRPOTrainerStep", "TreeRolloutBatch", "build_tree_rollout_batch", "compute_tree_advantage",
           "tree_dynamic_sampling_mask", "tree_grpo_loss", "tree_grpo_loss_from_logprobs", "tree_grpo_train_step"]

"""GRPO with vision/audio features held fixed per rollout batch
(reference: ``saint_llm_posttraining/multimodal_grpo_trainer.py:43-195``)."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.posttrain.grpo import (
    GRPOConfig,
    RolloutBatch,
    dynamic_sampling_mask,
    grpo_loss_from_logprobs,
    policy_token_logprobs,
)
from saint_llm_b200.posttrain.trainer import GRPOTrainerStep, frozen_logprobs


@dataclass(frozen=True)
class MultimodalRolloutBatch:
    tokens: Tensor
    response_mask: Tensor
    old_logprobs: Tensor
    ref_logprobs: Tensor
    rewards: Tensor
    vision_features: Tensor | None = None
    audio_features: Tensor | None = None

    def to_rollout_batch(self) -> RolloutBatch:
        return RolloutBatch(self.tokens, self.response_mask, self.old_logprobs, self.ref_logprobs, self.rewards)

    def features(self) -> dict[str, Tensor | None]:
        return {"vision_features": self.vision_features, "audio_features": self.audio_features}


def build_multimodal_rollout_batch(*, actor: nn.Module, ref: nn.Module | None, tokens: Tensor, response_mask: Tensor,
                                   rewards: Tensor, vision_features: Tensor | None = None,
                                   audio_features: Tensor | None = None) -> MultimodalRolloutBatch:
    feats = {"vision_features": vision_features, "audio_features": audio_features}
    old = frozen_logprobs(actor, tokens, **feats)
    refl = frozen_logprobs(ref, tokens, **feats) if ref is not None else old.clone()
    return MultimodalRolloutBatch(tokens, response_mask, old, refl, rewards, vision_features, audio_features)


def _select_feature_rows(feats: Tensor | None, slot_mask: Tensor, keep_rows: Tensor) -> Tensor | None:
    """Feature rows follow the slot tokens in row-major order; keep those of the kept rows."""
    if feats is None:
        return None
    owner = slot_mask.nonzero()[:, 0]  # row of every slot, in feature order
    return feats[keep_rows[owner]]


def select_rows(batch: MultimodalRolloutBatch, keep: Tensor, slots: object) -> MultimodalRolloutBatch:
    """Drop rows together with the feature rows of their placeholder slots."""
    idx = keep.nonzero().squeeze(-1)
    img = batch.tokens == slots.image_pad  # type: ignore[attr-defined]
    aud = (batch.tokens >= slots.audio_start) & (batch.tokens <= slots.audio_end)  # type: ignore[attr-defined]
    return MultimodalRolloutBatch(batch.tokens[idx], batch.response_mask[idx], batch.old_logprobs[idx],
                                  batch.ref_logprobs[idx], batch.rewards[idx],
                                  _select_feature_rows(batch.vision_features, img, keep),
                                  _select_feature_rows(batch.audio_features, aud, keep))


def multimodal_grpo_train_step(*, actor: nn.Module, optimizer: torch.optim.Optimizer, batch: MultimodalRolloutBatch,
                               cfg: GRPOConfig) -> GRPOTrainerStep:
    """Zero-variance groups are dropped together with their feature rows (the slot-to-feature
    alignment of the model's splice is kept)."""
    keep = dynamic_sampling_mask(batch.rewards, group_size=cfg.group_size)
    n_groups = int(keep.view(-1, cfg.group_size)[:, 0].sum())
    if n_groups == 0:
        zero = torch.zeros((), device=batch.rewards.device, requires_grad=True)
        return GRPOTrainerStep(zero, {"reward_mean": batch.rewards.mean().detach()}, 0)
    if n_groups * cfg.group_size != keep.numel():
        batch = select_rows(batch, keep, actor.cfg.tokenizer_slots)  # type: ignore[attr-defined]
    actor.train()
    lp = policy_token_logprobs(actor, batch.tokens, **batch.features())
    loss, metrics = grpo_loss_from_logprobs(lp, batch.to_rollout_batch(), cfg=cfg)
    optimizer.zero_grad(set_to_none=True)
    loss.backward()
    optimizer.step()
    return GRPOTrainerStep(loss.detach(), metrics, n_groups)


__all__ = ["MultimodalRolloutBatch", "build_multimodal_rollout_batch", "multimodal_grpo_train_step", "select_rows"]

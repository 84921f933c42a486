"""Specialist pipeline: SFT steps and GRPO steps from prompt strings and a reward function
around one actor/optimizer (reference: ``saint_llm_posttraining/specialist.py:74-231``)."""

from __future__ import annotations

import dataclasses
from collections.abc import Callable, Sequence
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.posttrain.grpo import GRPOConfig
from saint_llm_b200.posttrain.rollout import RolloutGenConfig, decode_rollouts_for_reward, generate_grpo_rollouts
from saint_llm_b200.posttrain.sft import SFTPackedBatch, sft_loss
from saint_llm_b200.posttrain.trainer import (
    GRPOTrainerStep,
    RewardFn,
    build_rollout_batch,
    grpo_train_step,
    score_rollouts,
)


@dataclass
class SFTStepOutput:
    loss: Tensor
    n_response_tokens: int


@dataclass
class RLStepOutput:
    train_step: GRPOTrainerStep
    rewards: Tensor
    n_rollouts: int


class SpecialistPipeline:
    def __init__(self, *, actor: nn.Module, ref: nn.Module | None, optimizer: torch.optim.Optimizer,
                 encode: Callable[[str], Sequence[int]], decode: Callable[[Sequence[int]], str],
                 eos_token: int | None = None, pad_token: int = 0) -> None:
        self.actor, self.ref, self.optimizer = actor, ref, optimizer
        self._encode, self._decode, self._eos, self._pad = encode, decode, eos_token, pad_token

    @property
    def device(self) -> torch.device:
        return next(self.actor.parameters()).device

    def sft_step(self, batch: SFTPackedBatch) -> SFTStepOutput:
        self.actor.train()
        loss = sft_loss(self.actor, batch.tokens.to(self.device), batch.loss_mask.to(self.device))
        self.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        self.optimizer.step()
        return SFTStepOutput(loss.detach(), int(batch.loss_mask[:, 1:].sum()))

    def encode_prompts(self, prompts: Sequence[str]) -> Tensor:
        """Right-padded (B, P) prompt ids."""
        ids = [list(self._encode(p)) for p in prompts]
        if not ids or any(not r for r in ids):
            raise ValueError("every prompt must encode to at least one token")
        out = torch.full((len(ids), max(map(len, ids))), self._pad, dtype=torch.long)
        for i, r in enumerate(ids):
            out[i, :len(r)] = torch.tensor(r)
        return out.to(self.device)

    def rl_step(self, prompts: Sequence[str], *, reward_fn: RewardFn, cfg: GRPOConfig,
                rollout_cfg: RolloutGenConfig) -> RLStepOutput:
        if not prompts:
            raise ValueError("prompts must be non-empty")
        if rollout_cfg.group_size != cfg.group_size:
            raise ValueError(f"rollout group_size {rollout_cfg.group_size} != GRPO group_size {cfg.group_size}")
        if rollout_cfg.eos_token is None and self._eos is not None:
            rollout_cfg = dataclasses.replace(rollout_cfg, eos_token=self._eos)
        prompt_ids = self.encode_prompts(prompts)
        self.actor.eval()
        tokens, mask = generate_grpo_rollouts(self.actor, prompt_ids, rollout_cfg)
        completions = decode_rollouts_for_reward(tokens, self._decode, prompt_len=prompt_ids.shape[1])
        rewards = score_rollouts(prompts=[p for p in prompts for _ in range(cfg.group_size)], completions=completions,
                                 reward_fn=reward_fn).to(tokens.device)
        batch = build_rollout_batch(actor=self.actor, ref=self.ref, tokens=tokens, response_mask=mask, rewards=rewards)
        step = grpo_train_step(actor=self.actor, optimizer=self.optimizer, batch=batch, cfg=cfg)
        return RLStepOutput(step, rewards.detach(), tokens.shape[0])


__all__ = ["RLStepOutput", "SFTStepOutput", "SpecialistPipeline"]

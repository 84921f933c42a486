"""Critique-GRPO helpers: pick low-reward rollouts, build critic and refinement prompts
(reference: ``saint_llm_posttraining/critique_grpo.py:46-194``; the prompt templates are
part of that recipe)."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from saint_llm_b200.posttrain.grpo import GRPOConfig


@dataclass(frozen=True)
class CritiqueGRPOConfig:
    grpo: GRPOConfig
    enabled: bool = False
    critique_threshold: float = 0.5
    critique_max_attempts: int = 1
    critic_self_play: bool = True


@dataclass(frozen=True)
class CritiqueRequest:
    rollout_idx: int
    original_prompt: str
    failed_completion: str
    reward: float


DEFAULT_CRITIQUE_TEMPLATE = (
    "The following completion received a low reward. Diagnose the specific reasoning error and explain what "
    "should have been done differently. Be brief — 2-3 sentences.\n\n"
    "Problem: {prompt}\nFailed completion: {completion}\nReward: {reward}\n\nCritique:"
)
DEFAULT_REFINEMENT_TEMPLATE = "{prompt}\n\nA previous attempt failed because: {critique}\n\nTry again, addressing the issue:"


def needs_critique_mask(rewards: Tensor, *, threshold: float) -> Tensor:
    return rewards < threshold


def make_critique_prompt(*, prompt: str, failed_completion: str, reward: float,
                         template: str = DEFAULT_CRITIQUE_TEMPLATE) -> str:
    return template.format(prompt=prompt, completion=failed_completion, reward=reward)


def make_refinement_prompt(*, prompt: str, critique: str, template: str = DEFAULT_REFINEMENT_TEMPLATE) -> str:
    return template.format(prompt=prompt, critique=critique)


def collect_critique_requests(*, rewards: Tensor, prompts: list[str], completions: list[str],
                              threshold: float) -> list[CritiqueRequest]:
    n = rewards.shape[0]
    if len(prompts) != n or len(completions) != n:
        raise ValueError(f"prompts ({len(prompts)}) / completions ({len(completions)}) must match rewards ({n})")
    vals = rewards.detach().float().cpu()
    idx = torch.nonzero(needs_critique_mask(vals, threshold=threshold)).flatten().tolist()
    return [CritiqueRequest(int(i), prompts[i], completions[i], float(vals[i])) for i in idx]


__all__ = ["DEFAULT_CRITIQUE_TEMPLATE", "DEFAULT_REFINEMENT_TEMPLATE", "CritiqueGRPOConfig", "CritiqueRequest",
           "collect_critique_requests", "make_critique_prompt", "make_refinement_prompt", "needs_critique_mask"]

"""Rollout generation for GRPO: G completions per prompt, ``(B*G, P + max_new)`` ids and
the response mask (reference: ``saint_llm_posttraining/rollout_generator.py:41-215``).
The mask covers the response through its first EOS.  Sampling decodes through the KV
cache (``use_cache``, default on)."""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Literal

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.generate import decode
from saint_llm_b200.infer.sampling import SamplingParams

SamplerKind = Literal["top_p", "greedy"]


@dataclass(frozen=True)
class RolloutGenConfig:
    group_size: int = 8
    max_new_tokens: int = 64
    sampler: SamplerKind = "top_p"
    temperature: float = 1.0
    top_p: float = 0.9
    eos_token: int | None = None
    pad_token: int = 0
    seed: int | None = None
    use_cache: bool = True


def response_mask_through_eos(tokens: Tensor, prompt_len: int, eos: int | None) -> Tensor:
    mask = torch.zeros_like(tokens)
    mask[:, prompt_len:] = 1
    if eos is not None:
        resp = tokens[:, prompt_len:] == eos
        after = (resp.cumsum(1) - resp.long()) > 0  # strictly after the first EOS
        mask[:, prompt_len:] = (~after).long()
    return mask


def _default_sampler(actor: nn.Module, prompt_ids: Tensor, cfg: RolloutGenConfig,
                     generator: torch.Generator | None) -> Tensor:
    if cfg.sampler not in ("top_p", "greedy"):
        raise ValueError(f"unknown sampler {cfg.sampler!r}")
    params = SamplingParams() if cfg.sampler == "greedy" else SamplingParams(temperature=cfg.temperature,
                                                                            top_p=cfg.top_p)
    return decode(actor, prompt_ids, max_new_tokens=cfg.max_new_tokens, params=params, eos_token=cfg.eos_token,
                  generator=generator, use_cache=cfg.use_cache)


@torch.no_grad()
def generate_grpo_rollouts(actor: nn.Module, prompt_ids: Tensor, cfg: RolloutGenConfig, *,
                           sampler: Callable[..., Tensor] | None = None) -> tuple[Tensor, Tensor]:
    if prompt_ids.dim() != 2:
        raise ValueError(f"prompt_ids must be 2D (B, P); got shape {tuple(prompt_ids.shape)}")
    if cfg.group_size <= 0 or cfg.max_new_tokens <= 0:
        raise ValueError("group_size and max_new_tokens must be positive")
    p = prompt_ids.shape[1]
    expanded = prompt_ids.repeat_interleave(cfg.group_size, dim=0)
    gen = torch.Generator(device=prompt_ids.device).manual_seed(cfg.seed) if cfg.seed is not None else None
    if sampler is not None:
        tokens = sampler(actor=actor, prompt_ids=expanded, cfg=cfg, generator=gen)
    else:
        tokens = _default_sampler(actor, expanded, cfg, gen)
    return tokens, response_mask_through_eos(tokens, p, cfg.eos_token)


def decode_rollouts_for_reward(tokens: Tensor, decode_fn: Callable[[list[int]], str], *,
                               prompt_len: int) -> list[str]:
    if tokens.dim() != 2:
        raise ValueError(f"tokens must be 2D (B*G, T); got shape {tuple(tokens.shape)}")
    if not 0 <= prompt_len <= tokens.shape[1]:
        raise ValueError(f"prompt_len {prompt_len} outside [0, {tokens.shape[1]}]")
    return [decode_fn(row) for row in tokens[:, prompt_len:].tolist()]


__all__ = ["RolloutGenConfig", "decode_rollouts_for_reward", "generate_grpo_rollouts", "response_mask_through_eos"]

"""Causal-LM perplexity (reference: ``saint_llm_eval/perplexity.py:24-86``): token-weighted
mean next-token CE in fp32, labels equal to ``ignore_index`` excluded, ``inf`` when nothing
is scored.  Per-token NLL comes from :func:`policy_token_logprobs` (fused LM-head kernel on
CUDA, no (B, T, V) logits)."""

from __future__ import annotations

import math
from collections.abc import Iterable

import torch
from torch import Tensor, nn


@torch.no_grad()
def token_nll(model: nn.Module, token_ids: Tensor, *, ignore_index: int = -100) -> tuple[Tensor, Tensor]:
    """(sum of NLL over scored positions, number of scored positions) as device scalars."""
    from saint_llm_b200.posttrain.grpo import policy_token_logprobs

    labels = token_ids[:, 1:]
    valid = labels != ignore_index
    safe = token_ids.clone()
    safe[:, 1:] = torch.where(valid, labels, torch.zeros_like(labels))
    lp = policy_token_logprobs(model, safe)[:, 1:].float()
    return -(lp * valid).sum(), valid.sum()


def _check(token_ids: Tensor) -> None:
    if token_ids.dim() != 2:
        raise ValueError(f"token_ids must be 2D (B, T); got {tuple(token_ids.shape)}")
    if token_ids.shape[1] < 2:
        raise ValueError(f"need at least 2 tokens to score; got T={token_ids.shape[1]}")


@torch.no_grad()
def compute_perplexity(model: nn.Module, token_ids: Tensor, *, ignore_index: int = -100) -> float:
    _check(token_ids)
    s, n = token_nll(model, token_ids, ignore_index=ignore_index)
    n_i = int(n)
    if n_i == 0 or not math.isfinite(float(s)):
        return math.inf
    return math.exp(float(s) / n_i)


@torch.no_grad()
def compute_perplexity_streaming(model: nn.Module, token_id_batches: Iterable[Tensor], *,
                                 ignore_index: int = -100) -> float:
    total, count = None, None
    for b in token_id_batches:
        if b.dim() != 2 or b.shape[1] < 2:
            continue
        s, n = token_nll(model, b, ignore_index=ignore_index)
        total = s if total is None else total + s
        count = n if count is None else count + n
    if count is None or int(count) == 0 or not math.isfinite(float(total)):
        return math.inf
    return math.exp(float(total) / int(count))


__all__ = ["compute_perplexity", "compute_perplexity_streaming", "token_nll"]

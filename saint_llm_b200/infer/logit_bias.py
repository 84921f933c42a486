"""Per-token additive logit bias (``{token_id: bias}``, the chat-API shape; reference:
``saint_llm_inference/logit_bias.py:27-67``)."""

from __future__ import annotations

from collections.abc import Mapping

from torch import Tensor

from saint_llm_b200.infer.sampling import bias_vector


def apply_logit_bias(logits: Tensor, bias: Mapping[int, float] | None) -> Tensor:
    vec = bias_vector(bias, logits.shape[-1], device=logits.device, dtype=logits.dtype)
    return logits if vec is None else logits + vec


def force_token_bias(token_id: int, *, magnitude: float = 1e9) -> dict[int, float]:
    return {int(token_id): float(magnitude)}


def forbid_tokens_bias(token_ids: list[int], *, magnitude: float = -1e9) -> dict[int, float]:
    return dict.fromkeys(map(int, token_ids), float(magnitude))


__all__ = ["apply_logit_bias", "forbid_tokens_bias", "force_token_bias"]

"""Multimodal prompt assembly and greedy decoding (reference:
``saint_llm_inference/multimodal_generate.py:49-142``).  Features are spliced during the
prefill; later steps decode from the KV cache (``use_cache=False`` recomputes every step
with the features, as the reference does)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.generate import decode
from saint_llm_b200.infer.sampling import SamplingParams


@dataclass(frozen=True)
class MultimodalSlots:
    image_pad: int
    audio_start: int
    audio_end: int


def build_multimodal_prompt_ids(text_ids_before: Sequence[int], text_ids_after: Sequence[int],
                                slots: MultimodalSlots, *, n_image_pads: int = 0, n_audio_tokens: int = 0,
                                device: torch.device | None = None) -> Tensor:
    """``before + image_pad * n + [audio_start, audio_start * n, audio_end] + after`` as (1, T)."""
    ids = list(text_ids_before) + [slots.image_pad] * n_image_pads
    if n_audio_tokens > 0:
        ids += [slots.audio_start] * (n_audio_tokens + 1) + [slots.audio_end]
    return torch.tensor([ids + list(text_ids_after)], dtype=torch.long, device=device)


def multimodal_greedy_decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int,
                             vision_features: Tensor | None = None, audio_features: Tensor | None = None,
                             eos_token: int | None = None, use_cache: bool = True) -> Tensor:
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, params=SamplingParams(), eos_token=eos_token,
                  use_cache=use_cache, vision_features=vision_features, audio_features=audio_features)


__all__ = ["MultimodalSlots", "build_multimodal_prompt_ids", "multimodal_greedy_decode"]

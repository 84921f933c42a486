"""Token-at-a-time generation for interactive use (reference:
``saint_llm_inference/streaming.py:50-206``): each yielded item is the ``(B, 1)`` next
ids; iteration stops when every row has produced EOS, every row has matched a stop
sequence, or after ``max_new_tokens``.

Unlike the reference, which re-runs the whole prefix every step, the stream decodes
through the KV cache by default (``use_cache=False`` restores full recomputation);
multimodal features are consumed by the prefill.
"""

from __future__ import annotations

from collections.abc import Iterator, Mapping, Sequence

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.kv_cache import KVCacheBundle
from saint_llm_b200.infer.generate import last_logits
from saint_llm_b200.infer.sampling import SamplingParams, bias_vector, next_token
from saint_llm_b200.infer.stop_sequences import StopSequenceMatcher


def _stream(model: nn.Module, prompt_ids: Tensor, params: SamplingParams, *, max_new_tokens: int,
            eos_token: int | None, generator: torch.Generator | None, stop_sequences: Sequence[Sequence[int]] | None,
            vision_features: Tensor | None, audio_features: Tensor | None, use_cache: bool) -> Iterator[Tensor]:
    if prompt_ids.dim() != 2:
        raise ValueError(f"prompt_ids must be 2D (B, T); got shape {tuple(prompt_ids.shape)}")
    if max_new_tokens <= 0:
        raise ValueError(f"max_new_tokens must be positive; got {max_new_tokens}")
    params.validate()
    b, t0 = prompt_ids.shape
    dev = prompt_ids.device
    ids = torch.empty((b, t0 + max_new_tokens), dtype=prompt_ids.dtype, device=dev)
    ids[:, :t0] = prompt_ids
    bundle = KVCacheBundle.for_model(model, max_seq_len=t0 + max_new_tokens, batch_size=b, device=dev) \
        if use_cache else None
    matchers = [StopSequenceMatcher(stop_sequences) for _ in range(b)] if stop_sequences else None
    seen = torch.zeros(b, dtype=torch.bool, device=dev)
    bias = None
    mm = {"vision_features": vision_features, "audio_features": audio_features}
    for i in range(max_new_tokens):
        cur = t0 + i
        if bundle is not None:
            logits = last_logits(model, ids[:, :cur] if i == 0 else ids[:, cur - 1:cur], bundle=bundle,
                                 **(mm if i == 0 else {}))
        else:
            logits = last_logits(model, ids[:, :cur], **mm)
        if bias is None and params.logit_bias:
            bias = bias_vector(params.logit_bias, logits.shape[-1], device=dev)
        tok = next_token(logits.float(), params, history=ids[:, :cur], generator=generator, bias=bias)
        ids[:, cur:cur + 1] = tok
        yield tok
        if eos_token is not None:
            seen |= tok.squeeze(-1) == eos_token
            if bool(seen.all()):
                return
        if matchers is not None:
            for m, t in zip(matchers, tok.squeeze(-1).tolist(), strict=True):
                m.feed(t)
            if all(m.matched() for m in matchers):
                return


@torch.no_grad()
def stream_greedy_decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, eos_token: int | None = None,
                         stop_sequences: Sequence[Sequence[int]] | None = None,
                         vision_features: Tensor | None = None, audio_features: Tensor | None = None,
                         logit_bias: Mapping[int, float] | None = None, use_cache: bool = True) -> Iterator[Tensor]:
    yield from _stream(model, prompt_ids, SamplingParams(logit_bias=logit_bias), max_new_tokens=max_new_tokens,
                       eos_token=eos_token, generator=None, stop_sequences=stop_sequences,
                       vision_features=vision_features, audio_features=audio_features, use_cache=use_cache)


@torch.no_grad()
def stream_top_p_sample(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, p: float = 0.9,
                        temperature: float = 1.0, top_k: int | None = None, eos_token: int | None = None,
                        generator: torch.Generator | None = None, stop_sequences: Sequence[Sequence[int]] | None = None,
                        vision_features: Tensor | None = None, audio_features: Tensor | None = None,
                        logit_bias: Mapping[int, float] | None = None, use_cache: bool = True) -> Iterator[Tensor]:
    params = SamplingParams(temperature=temperature, top_k=top_k, top_p=p, logit_bias=logit_bias)
    yield from _stream(model, prompt_ids, params, max_new_tokens=max_new_tokens, eos_token=eos_token,
                       generator=generator, stop_sequences=stop_sequences, vision_features=vision_features,
                       audio_features=audio_features, use_cache=use_cache)


__all__ = ["stream_greedy_decode", "stream_top_p_sample"]

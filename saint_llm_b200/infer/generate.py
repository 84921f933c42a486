"""Decoding loops: greedy / top-k / top-p, with or without the KV cache.

Public functions and their output contract are the reference's
(``saint_llm_inference/generate.py:22-476``): ``(B, T + max_new_tokens)`` ids; with
``eos_token`` set, once every row has produced EOS the remaining positions are EOS.

One engine (:func:`decode`) runs all of them.  Differences from a per-step Python loop:

* output ids go into one preallocated buffer (no ``torch.cat`` per step);
* the all-rows-finished test never blocks the device: after the step at which every
  row has seen EOS, further tokens are forced to EOS on the device, and the host looks
  at the flag only every ``sync_every`` steps to stop early.  The produced ids equal
  the stop-immediately loop's;
* only the last position's logits are computed (the LM head runs on ``(B, 1, D)``, not
  ``(B, T, D)``), and the MTP / generation heads are skipped.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.kv_cache import KVCacheBundle
from saint_llm_b200.infer.sampling import SamplingParams, bias_vector, next_token


def last_logits(model: nn.Module, ids: Tensor, *, bundle: KVCacheBundle | None = None,
                vision_features: Tensor | None = None, audio_features: Tensor | None = None) -> Tensor:
    """(B, V) logits of the last position."""
    if hasattr(model, "backbone") and hasattr(model, "logits"):
        h, _ = model.backbone(ids, vision_features, audio_features, kv_cache_bundle=bundle)
        return model.logits(h[:, -1:]).squeeze(1)
    kw = {k: v for k, v in (("vision_features", vision_features), ("audio_features", audio_features))
          if v is not None}
    if bundle is not None:
        kw["kv_cache_bundle"] = bundle
    return model(ids, **kw)["logits"][:, -1]


@torch.no_grad()
def decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, params: SamplingParams,
           eos_token: int | None = None, generator: torch.Generator | None = None, use_cache: bool = False,
           bundle: KVCacheBundle | None = None, draw: str = "full", vision_features: Tensor | None = None,
           audio_features: Tensor | None = None, sync_every: int = 8,
           on_token: Callable[[Tensor], bool] | None = None) -> Tensor:
    """Generate ``max_new_tokens`` ids after ``prompt_ids``; see the module docstring."""
    if prompt_ids.dim() != 2:
        raise ValueError(f"prompt_ids must be 2D (B, T); got shape {tuple(prompt_ids.shape)}")
    params.validate()
    b, t0 = prompt_ids.shape
    dev = prompt_ids.device
    out = torch.full((b, t0 + max_new_tokens), eos_token if eos_token is not None else 0, dtype=prompt_ids.dtype,
                     device=dev)
    out[:, :t0] = prompt_ids
    if max_new_tokens <= 0:
        return out
    if use_cache and bundle is None:
        bundle = KVCacheBundle.for_model(model, max_seq_len=t0 + max_new_tokens, batch_size=b, device=dev)
    bias = None
    seen = torch.zeros(b, dtype=torch.bool, device=dev)
    finished = torch.zeros((), dtype=torch.bool, device=dev)
    mm = {"vision_features": vision_features, "audio_features": audio_features}
    for i in range(max_new_tokens):
        cur = t0 + i
        if use_cache:
            step_ids = out[:, :cur] if i == 0 else out[:, cur - 1:cur]
            logits = last_logits(model, step_ids, bundle=bundle, **(mm if i == 0 else {}))
        else:
            logits = last_logits(model, out[:, :cur], **mm)
        if bias is None and params.logit_bias:
            bias = bias_vector(params.logit_bias, logits.shape[-1], device=dev, dtype=torch.float32)
        tok = next_token(logits.float(), params, history=out[:, :cur], generator=generator, bias=bias, draw=draw)
        if eos_token is not None:
            tok = torch.where(finished, torch.full_like(tok, eos_token), tok)
            seen |= tok.squeeze(-1) == eos_token
            finished |= seen.all()
        out[:, cur:cur + 1] = tok
        if on_token is not None and on_token(tok):
            break
        if eos_token is not None and ((i + 1) % sync_every == 0 or i == 0) and bool(finished):
            break
    return out


def _check_k(k: int) -> None:
    if k <= 0:
        raise ValueError(f"k must be positive; got {k}")


def greedy_decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int,
                  eos_token: int | None = None) -> Tensor:
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, params=SamplingParams(), eos_token=eos_token)


def greedy_decode_cached(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, eos_token: int | None = None,
                         bundle: KVCacheBundle | None = None) -> Tensor:
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, params=SamplingParams(), eos_token=eos_token,
                  use_cache=True, bundle=bundle)


def top_k_sample(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, k: int = 50,
                 temperature: float = 1.0, eos_token: int | None = None, generator: torch.Generator | None = None,
                 repetition_penalty: float | None = None) -> Tensor:
    _check_k(k)
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, eos_token=eos_token, generator=generator,
                  params=SamplingParams(temperature=temperature, top_k=k, repetition_penalty=repetition_penalty),
                  draw="topk")


def top_k_sample_cached(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, k: int = 50,
                        temperature: float = 1.0, eos_token: int | None = None,
                        generator: torch.Generator | None = None, bundle: KVCacheBundle | None = None,
                        repetition_penalty: float | None = None) -> Tensor:
    _check_k(k)
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, eos_token=eos_token, generator=generator,
                  params=SamplingParams(temperature=temperature, top_k=k, repetition_penalty=repetition_penalty),
                  draw="topk", use_cache=True, bundle=bundle)


def top_p_sample(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, p: float = 0.9,
                 temperature: float = 1.0, top_k: int | None = None, eos_token: int | None = None,
                 generator: torch.Generator | None = None, repetition_penalty: float | None = None) -> Tensor:
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, eos_token=eos_token, generator=generator,
                  params=SamplingParams(temperature=temperature, top_k=top_k, top_p=p,
                                        repetition_penalty=repetition_penalty))


def top_p_sample_cached(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, p: float = 0.9,
                        temperature: float = 1.0, top_k: int | None = None, eos_token: int | None = None,
                        generator: torch.Generator | None = None, bundle: KVCacheBundle | None = None,
                        repetition_penalty: float | None = None) -> Tensor:
    return decode(model, prompt_ids, max_new_tokens=max_new_tokens, eos_token=eos_token, generator=generator,
                  params=SamplingParams(temperature=temperature, top_k=top_k, top_p=p,
                                        repetition_penalty=repetition_penalty), use_cache=True, bundle=bundle)


__all__ = ["decode", "greedy_decode", "greedy_decode_cached", "last_logits", "top_k_sample", "top_k_sample_cached",
           "top_p_sample", "top_p_sample_cached"]

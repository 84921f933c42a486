"""Next-token selection: temperature, repetition penalty, logit bias, top-k, top-p.

Semantics follow the reference's decoders (``saint_llm_inference/generate.py:271-323``,
``logit_bias.py:27-67``): HF-style repetition penalty (positive logits divided, negative
multiplied, over the ids present in the history), a top-p nucleus that always keeps the
best token and is the smallest prefix whose mass reaches ``p``, top-k as a cutoff at the
k-th largest logit (ties kept), and sampling by ``torch.multinomial`` so a seeded
generator reproduces a run.  Everything stays on the device (no host round trips).

On CUDA, bias, temperature, top-k, top-p and the draw run as one native kernel per call
(``csrc/sampling.cu``: radix selection of the top-k / top-p thresholds, inverse-CDF draw
against a uniform from the caller's generator); the PyTorch functions below are its
oracle and the CPU path.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0           # < 1e-8 means greedy
    top_k: int | None = None
    top_p: float = 1.0
    repetition_penalty: float | None = None
    logit_bias: Mapping[int, float] | None = None

    def validate(self) -> None:
        if self.temperature < 0.0:
            raise ValueError(f"temperature must be >= 0; got {self.temperature}")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError(f"p must be in (0, 1]; got {self.top_p}")
        if self.top_k is not None and self.top_k <= 0:
            raise ValueError(f"top_k must be positive when set; got {self.top_k}")
        if self.repetition_penalty is not None and self.repetition_penalty <= 0.0:
            raise ValueError(f"repetition_penalty must be > 0 when set; got {self.repetition_penalty}")

    @property
    def greedy(self) -> bool:
        return self.temperature < 1.0e-8


def apply_repetition_penalty(logits: Tensor, history: Tensor, penalty: float) -> Tensor:
    if penalty == 1.0:
        return logits
    seen = torch.gather(logits, -1, history)
    return logits.scatter(-1, history, torch.where(seen > 0, seen / penalty, seen * penalty))


def bias_vector(bias: Mapping[int, float] | None, vocab: int, *, device: torch.device | None = None,
                dtype: torch.dtype = torch.float32) -> Tensor | None:
    """Dense (V,) bias from a ``{token_id: value}`` map; ids outside the vocabulary are ignored."""
    if not bias:
        return None
    items = [(int(k), float(v)) for k, v in bias.items() if 0 <= int(k) < vocab]
    vec = torch.zeros(vocab, dtype=dtype)
    if items:
        idx, val = zip(*items, strict=True)
        vec[list(idx)] = torch.tensor(val, dtype=dtype)
    return vec.to(device)


def filter_top_k(logits: Tensor, k: int) -> Tensor:
    kth = logits.topk(min(k, logits.shape[-1]), dim=-1).values[..., -1:]
    return logits.masked_fill(logits < kth, float("-inf"))


def filter_top_p(logits: Tensor, p: float) -> Tensor:
    srt, order = logits.sort(dim=-1, descending=True)
    probs = torch.softmax(srt, dim=-1)
    keep_sorted = (probs.cumsum(-1) - probs) <= p
    keep_sorted[..., 0] = True
    keep = torch.empty_like(keep_sorted).scatter_(-1, order, keep_sorted)
    return logits.masked_fill(~keep, float("-inf"))


def sample_from_topk(logits: Tensor, k: int, generator: torch.Generator | None) -> Tensor:
    """Sample among the k best logits (the reference's ``top_k_sample`` draw)."""
    vals, idx = logits.topk(min(k, logits.shape[-1]), dim=-1)
    pick = torch.multinomial(torch.softmax(vals, dim=-1), 1, generator=generator)
    return idx.gather(-1, pick)


def fused_sample(logits: Tensor, *, temperature: float, top_k: int | None = None, top_p: float = 1.0,
                 bias: Tensor | None = None, generator: torch.Generator | None = None,
                 return_threshold: bool = False) -> Tensor | tuple[Tensor, Tensor]:
    """(B, V) logits -> (B, 1) token ids in one native kernel (CUDA only).

    The uniform of each row comes from ``generator`` (torch.rand), so a seeded generator
    reproduces the draws.  ``return_threshold`` also returns the order-preserving integer
    key of the smallest kept logit per row (for testing the kept set)."""
    from saint_llm_b200.ops import backend

    b = logits.shape[0]
    x = logits if logits.dtype in (torch.float32, torch.bfloat16) else logits.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    gdev = generator.device if generator is not None else x.device
    u = torch.rand(b, generator=generator, device=gdev, dtype=torch.float32).to(x.device, non_blocking=True)
    out = torch.empty(b, dtype=torch.long, device=x.device)
    thr = torch.empty(b, dtype=torch.int32, device=x.device) if return_threshold else None
    bv = None if bias is None else bias.float().contiguous()
    backend.ext().sample_tokens(x, bv, float(temperature), int(top_k or 0), float(top_p), u, out, thr)
    return (out.view(b, 1), thr) if return_threshold else out.view(b, 1)


def next_token(last_logits: Tensor, params: SamplingParams, *, history: Tensor | None = None,
               generator: torch.Generator | None = None, bias: Tensor | None = None,
               draw: str = "full") -> Tensor:
    """(B, V) logits -> (B, 1) token ids.

    ``draw="topk"`` samples within the top-k set directly (``top_k_sample`` semantics);
    ``"full"`` masks then samples from the full softmax (``top_p_sample`` semantics).
    """
    from saint_llm_b200.ops import backend

    if backend.native_for(last_logits) and last_logits.dim() == 2:
        x = last_logits
        if params.repetition_penalty is not None and history is not None and not params.greedy:
            # the penalty rescales by sign, so it commutes with the temperature division
            x = apply_repetition_penalty(x.float(), history, params.repetition_penalty)
        k = params.top_k if draw == "full" else (params.top_k or x.shape[-1])
        return fused_sample(x, temperature=0.0 if params.greedy else params.temperature, top_k=k,
                            top_p=params.top_p if draw == "full" else 1.0, bias=bias, generator=generator)
    x = last_logits
    if bias is not None:
        x = x + bias.to(x.dtype)
    if params.greedy:
        return x.argmax(dim=-1, keepdim=True)
    x = x / params.temperature
    if params.repetition_penalty is not None and history is not None:
        x = apply_repetition_penalty(x, history, params.repetition_penalty)
    if draw == "topk":
        return sample_from_topk(x, params.top_k or x.shape[-1], generator)
    if params.top_k is not None:
        x = filter_top_k(x, params.top_k)
    if params.top_p < 1.0:
        x = filter_top_p(x, params.top_p)
    return torch.multinomial(torch.softmax(x, dim=-1), 1, generator=generator)


__all__ = ["SamplingParams", "apply_repetition_penalty", "bias_vector", "filter_top_k", "filter_top_p",
           "fused_sample", "next_token", "sample_from_topk"]

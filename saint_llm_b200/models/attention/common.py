"""Attention primitives shared by SWA / CSA / HCA / NSA.

Semantics follow the reference exactly (``core/attention/common.py:12-124``):

* ``RMSNorm``: ``w * x * rsqrt(mean(x^2) + eps)`` in the input dtype.
* Partial RoPE rotates the *last* ``rope_dim`` channels with *interleaved* pairs
  ``(x[0::2], x[1::2])``; the leading channels pass through.
* ``attend`` computes ``softmax(QK^T/sqrt(d))V`` with an optional per-head sink logit
  that only enlarges the softmax denominator, an optional Gemma softcap applied after
  the score observer (MuonClip telemetry sees the uncapped score) and a boolean
  visibility mask.

On CUDA the model never calls ``attend`` on a training path (the fused sm_100a
kernels in ``saint_llm_b200.ops.attention`` replace it); it is the oracle.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch
from torch import Tensor, nn


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1.0e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        from saint_llm_b200.ops import backend

        if backend.native_for(x) and x.shape[-1] % 8 == 0:
            from saint_llm_b200.ops.norm import rms_norm

            return rms_norm(x, self.weight, self.eps)
        return self.weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps))


def rope_tables(n_pos: int, rope_dim: int, theta: float = 10000.0,
                device: torch.device | None = None, start: int = 0) -> tuple[Tensor, Tensor]:
    """cos/sin tables of shape (n_pos, rope_dim/2) for positions ``start .. start+n_pos-1``."""
    if rope_dim % 2:
        raise ValueError("RoPE needs an even rotary dimension")
    exponent = torch.arange(0, rope_dim, 2, device=device, dtype=torch.float32) / rope_dim
    inv_freq = 1.0 / (theta ** exponent)
    pos = torch.arange(start, start + n_pos, device=device, dtype=torch.float32)
    ang = pos[:, None] * inv_freq[None, :]
    return ang.cos(), ang.sin()


# Reference-compatible name (``build_rope_cache(seq_len, head_dim, base, device)``).
def build_rope_cache(seq_len: int, head_dim: int, base: float = 10000.0,
                     device: torch.device | None = None) -> tuple[Tensor, Tensor]:
    return rope_tables(seq_len, head_dim, base, device)


def apply_partial_rope(x: Tensor, cos: Tensor, sin: Tensor, rope_dim: int) -> Tensor:
    """Rotate the last ``rope_dim`` channels of ``x`` (..., T, D) with interleaved pairs."""
    if rope_dim == 0:
        return x
    d = x.shape[-1]
    if rope_dim > d:
        raise ValueError("rope_dim exceeds head_dim")
    rot = x[..., d - rope_dim:]
    even, odd = rot[..., 0::2], rot[..., 1::2]
    shape = (1,) * (even.dim() - cos.dim()) + tuple(cos.shape)
    c, s = cos.reshape(shape), sin.reshape(shape)
    out = torch.stack((even * c - odd * s, even * s + odd * c), dim=-1).flatten(-2)
    if rope_dim == d:
        return out
    return torch.cat([x[..., : d - rope_dim], out], dim=-1)


def causal_mask(t_q: int, t_k: int, device: torch.device | None = None) -> Tensor:
    """True where key j is visible from query i (right-aligned when t_k > t_q)."""
    qi = torch.arange(t_q, device=device)[:, None] + (t_k - t_q)
    return torch.arange(t_k, device=device)[None, :] <= qi


def sliding_window_mask(t: int, window: int, device: torch.device | None = None) -> Tensor:
    """True where 0 <= i - j < window (square)."""
    diff = torch.arange(t, device=device)[:, None] - torch.arange(t, device=device)[None, :]
    return (diff >= 0) & (diff < window)


def window_mask_at(q_start: int, n_q: int, n_k: int, window: int,
                   device: torch.device | None = None) -> Tensor:
    """Causal sliding-window mask for queries at absolute positions q_start.. vs keys 0..n_k-1."""
    qp = torch.arange(q_start, q_start + n_q, device=device)[:, None]
    kp = torch.arange(n_k, device=device)[None, :]
    return (kp <= qp) & (qp - kp < window)


def softmax_with_sink(scores: Tensor, sink_logit: Tensor | None) -> Tensor:
    """Softmax over the last dim with ``exp(sink_h)`` added to each head's denominator.

    ``scores`` is (..., H, Tq, Tk); ``sink_logit`` is (H,).
    """
    if sink_logit is None:
        return torch.softmax(scores, dim=-1)
    sink = sink_logit.reshape((1,) * (scores.dim() - 3) + (-1, 1, 1)).to(scores.dtype)
    sink = sink.expand(*scores.shape[:-1], 1)
    return torch.softmax(torch.cat([scores, sink], dim=-1), dim=-1)[..., :-1]


def scaled_dot_product(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    mask: Tensor | None = None,
    sink_logit: Tensor | None = None,
    score_observer: Callable[[Tensor], None] | None = None,
    logit_softcap: float | None = None,
) -> Tensor:
    """Dense attention oracle. q (B,H,Tq,d); k, v (B,H|1,Tk,d).

    With one K/V head (MQA) the heads are folded into the query rows, (B, H*Tq, d) x
    (B, d, Tk), so the shared K/V are never broadcast-copied per head."""
    b, h, tq, d = q.shape
    mqa = k.shape[1] == 1 and h > 1 and k.shape[0] == b and v.shape[0] == b
    if mqa:
        scores = torch.bmm(q.reshape(b, h * tq, d), k[:, 0].transpose(-1, -2)).view(b, h, tq, -1)
        scores = scores / math.sqrt(d)
    else:
        scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if score_observer is not None:
        score_observer(scores)
    if logit_softcap is not None:
        scores = logit_softcap * torch.tanh(scores / logit_softcap)
    if mask is not None:
        scores = scores.masked_fill(~mask, float("-inf"))
    p = softmax_with_sink(scores, sink_logit)
    if mqa:
        return torch.bmm(p.reshape(b, h * tq, -1).to(v.dtype), v[:, 0]).view(b, h, tq, v.shape[-1])
    return torch.matmul(p, v)


attend = scaled_dot_product

__all__ = [
    "RMSNorm",
    "apply_partial_rope",
    "attend",
    "build_rope_cache",
    "causal_mask",
    "rope_tables",
    "scaled_dot_product",
    "sliding_window_mask",
    "softmax_with_sink",
    "window_mask_at",
]

"""Tree attention: attention over K/V split into chunks (or ranks), combined with the
associative log-sum-exp merge of partial results (reference
``core/attention/tree_attention.py:39-126``, which runs the chunks in one process only).

A partial over a key subset is ``(m, l, o)``: row max of the scores, sum of
``exp(s - m)`` and the normalised output.  Two partials merge as
``m = max(m_a, m_b)``, ``l = e^(m_a-m) l_a + e^(m_b-m) l_b``,
``o = (e^(m_a-m) l_a o_a + e^(m_b-m) l_b o_b) / l``.

``tree_attention`` walks local chunks; ``tree_attention_distributed`` is the
sequence-parallel form: each rank holds a K/V shard, computes its partial, and two
all-reduces (MAX of ``m``, then SUM of the rescaled ``l`` and ``l*o``) give every rank the
exact result.  ``merge_partials`` is the same merge for split-K decode.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor


def attention_partial(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None = None,
                      scale: float | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """fp32 ``(m, l, o)`` over the given keys; fully masked rows give m=-inf, l=0, o=0."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    m = s.amax(-1)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m_safe.unsqueeze(-1))
    l = p.sum(-1)  # noqa: E741
    o = torch.matmul(p, v.float()) / l.clamp(min=1e-30).unsqueeze(-1)
    return m, l, o


def merge_partials(parts: list[tuple[Tensor, Tensor, Tensor]]) -> tuple[Tensor, Tensor, Tensor]:
    """Merge partials ``(m, l, o)``; on CUDA one ``lse_merge`` kernel (``ops.decode``)."""
    from saint_llm_b200.ops import backend

    if parts and backend.native_for(parts[0][2]):
        from saint_llm_b200.ops.decode import lse_merge

        return lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                         torch.stack([p[2] for p in parts]))
    m = torch.stack([p[0] for p in parts]).amax(0)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    l = torch.zeros_like(m)  # noqa: E741
    acc = torch.zeros_like(parts[0][2])
    for mi, li, oi in parts:
        w = torch.exp(mi - m_safe) * li
        w = torch.where(li > 0, w, torch.zeros_like(w))
        l = l + w  # noqa: E741
        acc = acc + w.unsqueeze(-1) * oi
    return m, l, acc / l.clamp(min=1e-30).unsqueeze(-1)


def _check(q: Tensor, k: Tensor, v: Tensor) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"q/k/v must be 4-D (B, H, T, D); got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if k.shape != v.shape:
        raise ValueError(f"k and v must share shape; got {tuple(k.shape)} vs {tuple(v.shape)}")
    if q.shape[:2] != k.shape[:2]:
        raise ValueError(f"q and k must agree on (B, H); got {tuple(q.shape[:2])} vs {tuple(k.shape[:2])}")


def tree_attention(q: Tensor, k: Tensor, v: Tensor, *, n_chunks: int = 1, mask: Tensor | None = None) -> Tensor:
    """Dense-equivalent attention computed over ``n_chunks`` K/V chunks; rows with no visible
    key output zero.  ``mask`` is (Tq, Tk) bool, True = visible."""
    _check(q, k, v)
    if n_chunks <= 0:
        raise ValueError(f"n_chunks must be positive; got {n_chunks}")
    tk = k.shape[-2]
    step = max(1, math.ceil(tk / n_chunks))
    parts = [attention_partial(q, k[..., s:s + step, :], v[..., s:s + step, :],
                               None if mask is None else mask[:, s:s + step]) for s in range(0, tk, step)]
    _, l, o = merge_partials(parts)  # noqa: E741
    return torch.where((l > 0).unsqueeze(-1), o, torch.zeros_like(o)).to(q.dtype)


def tree_attention_distributed(q: Tensor, k_local: Tensor, v_local: Tensor, *, mask_local: Tensor | None = None,
                               group: dist.ProcessGroup | None = None) -> Tensor:
    """Every rank holds all queries and its own K/V shard; returns the full attention output."""
    m, l, o = attention_partial(q, k_local, v_local, mask_local)  # noqa: E741
    m_g = m.clone()
    dist.all_reduce(m_g, op=dist.ReduceOp.MAX, group=group)
    m_safe = torch.where(torch.isfinite(m_g), m_g, torch.zeros_like(m_g))
    w = torch.where(l > 0, torch.exp(m - m_safe) * l, torch.zeros_like(l))
    packed = torch.cat([w.unsqueeze(-1), w.unsqueeze(-1) * o], dim=-1)
    dist.all_reduce(packed, op=dist.ReduceOp.SUM, group=group)
    l_g, acc = packed[..., 0], packed[..., 1:]
    out = acc / l_g.clamp(min=1e-30).unsqueeze(-1)
    return torch.where((l_g > 0).unsqueeze(-1), out, torch.zeros_like(out)).to(q.dtype)


__all__ = ["attention_partial", "merge_partials", "tree_attention", "tree_attention_distributed"]

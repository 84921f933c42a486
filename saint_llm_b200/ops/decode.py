"""Native single-token decode attention over the heterogeneous cache (one kernel per layer).

``decode_attention`` computes, for every sequence and query head, the sliding-window
branch (ring of W slots, live iff the slot's age is <= pos, softcap, optional sink) plus
the compressed branch (HCA: every visible entry, optional sink; CSA: the listed top-k
entries), with K = V = RMSNorm(entry) applied on the fly.  The eager composition it
replaces is ``infer.static_decode._attend_layer_eager``.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from saint_llm_b200.ops import backend


def supported(head_dim: int, heads: int) -> bool:
    return head_dim == 128 and heads % 4 == 0


def decode_attention(q: Tensor, k_win: Tensor, v_win: Tensor, pos: Tensor, *, sink: Tensor | None,
                     softcap: float | None, mode: int = 0, entries: Tensor | None = None,
                     norm_weight: Tensor | None = None, norm_eps: float = 1e-6, m: int = 0,
                     top: Tensor | None = None, comp_sink: Tensor | None = None) -> Tensor:
    """q (B, H, 1, 128); k_win / v_win (B, W, 128); pos: int64 device scalar.
    mode 0: window only; 1: + HCA entries (B, n, 128) with compression rate ``m``;
    2: + CSA entries gathered by ``top`` (B, k) int64 (-1 = none).  Returns (B, H, 1, 128)."""
    b, h, _, d = q.shape
    out = torch.empty(b, h, 1, d, dtype=torch.bfloat16, device=q.device)
    backend.ext().decode_attention(
        q.reshape(b, h, d).to(torch.bfloat16).contiguous(), k_win, v_win, pos,
        None if sink is None else sink.float().contiguous(), float(softcap or 0.0), mode,
        entries, None if norm_weight is None else norm_weight.float().contiguous(), float(norm_eps), int(m),
        None if top is None else top.reshape(b, -1).contiguous(),
        None if comp_sink is None else comp_sink.float().contiguous(), 1.0 / math.sqrt(d), out)
    return out


__all__ = ["decode_attention", "supported"]

"""Native Sparse Attention (NSA, arXiv 2502.11089), opt-in alternative to the CSA/HCA/SWA
interleave (reference ``core/attention/nsa.py:70-294``).

Three branches over one MQA K/V head, mixed per token and head by a zero-initialised
sigmoid gate normalised over the branches (1/3 each at init):

* compressed: mean-pooled K/V blocks of ``compression_rate`` tokens; block ``i`` is
  visible to query ``t`` iff ``(i+1)*m - 1 <= t``; sink and softcap as in SWA; rows with
  no visible block output zero;
* selective: per (batch, head, query) the ``selection_k`` visible blocks whose pooled
  key scores highest; attention over those blocks' raw tokens (no sink);
* sliding window: the SWA branch.

The reference selects tokens with a per-(b, h, t) Python loop.  Here the selection is a
boolean block mask scattered from ``topk`` and expanded to tokens, evaluated in query
chunks, so the cost is a few batched matmuls.  With a KV cache (the window cache keeps
the whole post-RoPE history) the branches are recomputed over the cached K/V, so NSA
also decodes incrementally; the reference ignores the cache argument.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import Tensor, nn

from saint_llm_b200.config import AttentionConfig
from saint_llm_b200.models.attention.common import scaled_dot_product, window_mask_at
from saint_llm_b200.models.attention.csa import _AttentionBase
from saint_llm_b200.models.linear import LinearFactory, default_linear


def block_compress(x: Tensor, *, block_size: int) -> Tensor:
    """Mean-pool ``(..., T, D)`` into ``(..., T // block_size, D)``; the tail is dropped."""
    n = x.shape[-2] // block_size if block_size > 0 else 0
    if n == 0:
        return x.new_zeros(*x.shape[:-2], 0, x.shape[-1])
    return x[..., :n * block_size, :].unflatten(-2, (n, block_size)).mean(-2)


def selective_attention(q: Tensor, k: Tensor, v: Tensor, *, block_size: int, top_k: int, q_start: int = 0,
                        logit_softcap: float | None = None, query_chunk: int = 512) -> Tensor:
    """q (B, H, Tq, d) at absolute positions ``q_start..``; k, v (B, Tk, d) (one KV head)."""
    b, h, tq, d = q.shape
    nb = k.shape[1] // block_size
    if nb == 0 or top_k <= 0:
        return torch.zeros_like(q)
    kk = min(top_k, nb)
    scale = 1.0 / math.sqrt(d)
    kc = block_compress(k, block_size=block_size).unsqueeze(1)            # (B, 1, nb, d)
    kt = k[:, :nb * block_size].unsqueeze(1)                                # (B, 1, nb*m, d)
    vt = v[:, :nb * block_size].unsqueeze(1)
    block_end = (torch.arange(nb, device=q.device) + 1) * block_size - 1
    outs = []
    for s in range(0, tq, query_chunk):
        qc = q[:, :, s:s + query_chunk]
        pos = torch.arange(q_start + s, q_start + s + qc.shape[2], device=q.device)
        visible = block_end[None, :] <= pos[:, None]                        # (tc, nb)
        bscore = torch.matmul(qc, kc.transpose(-1, -2)) * scale
        bscore = bscore.masked_fill(~visible, float("-inf"))
        pick = torch.zeros_like(bscore, dtype=torch.bool).scatter_(-1, bscore.topk(kk, dim=-1).indices, True)
        tok = (pick & visible).repeat_interleave(block_size, dim=-1)       # (B, H, tc, nb*m)
        sc = torch.matmul(qc, kt.transpose(-1, -2)) * scale
        if logit_softcap is not None:
            sc = logit_softcap * torch.tanh(sc / logit_softcap)
        any_tok = tok.any(-1, keepdim=True)
        sc = sc.masked_fill(~tok, float("-inf")).masked_fill(~any_tok, 0.0)
        outs.append(torch.matmul(torch.softmax(sc, dim=-1), vt) * any_tok)
    return torch.cat(outs, dim=2)


class NSAttention(_AttentionBase):
    """Parameter names match the reference module (checkpoint compatible)."""

    def __init__(self, hidden_dim: int, attn: AttentionConfig, *, compression_rate: int = 32, selection_k: int = 16,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__(hidden_dim, attn, linear_factory=linear_factory)
        self.compression_rate, self.selection_k = compression_rate, selection_k
        self.k_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.v_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.branch_gate = nn.Linear(attn.head_dim, 3, bias=True)
        nn.init.zeros_(self.branch_gate.weight)
        nn.init.zeros_(self.branch_gate.bias)
        self._finish_init(hidden_dim, attn, linear_factory)

    def _observe(self, scores: Tensor) -> None:
        m = scores.detach().abs().amax().to(self.max_attn_logit.dtype)
        self.max_attn_logit.copy_(torch.maximum(self.max_attn_logit, m))

    def compressed_branch(self, q: Tensor, k: Tensor, v: Tensor, q_start: int) -> Tensor:
        cr = self.compression_rate
        kc, vc = block_compress(k, block_size=cr), block_compress(v, block_size=cr)
        nb = kc.shape[1]
        if nb == 0:
            return torch.zeros_like(q)
        pos = torch.arange(q_start, q_start + q.shape[2], device=q.device)[:, None]
        visible = (torch.arange(nb, device=q.device)[None, :] + 1) * cr - 1 <= pos
        any_blk = visible.any(-1, keepdim=True)
        out = scaled_dot_product(q, kc.unsqueeze(1), vc.unsqueeze(1), mask=visible | ~any_blk,
                                 sink_logit=self.sink_logit, score_observer=self._observe,
                                 logit_softcap=self.attn_cfg.logit_softcap)
        return out * any_blk.view(1, 1, -1, 1)

    def forward(self, h: Tensor, is_visual: Tensor | None = None, *, kv_cache: Any | None = None) -> Tensor:
        del is_visual  # NSA has no visual block bias
        cfg = self.attn_cfg
        self.max_attn_logit.zero_()
        off, cos, sin = self._positions(h, kv_cache)
        q = self._queries(h, cos, sin)
        k, v = self._sw_kv(h, cos, sin)
        if kv_cache is not None:
            k, v = kv_cache.append(k, v)
        comp = self.compressed_branch(q, k, v, off)
        sel = selective_attention(q, k, v, block_size=self.compression_rate, top_k=self.selection_k, q_start=off,
                                  logit_softcap=cfg.logit_softcap)
        lo = max(0, off - cfg.sliding_window_size + 1) if k.shape[1] > q.shape[2] else 0
        mask = window_mask_at(off - lo, q.shape[2], k.shape[1] - lo, cfg.sliding_window_size, q.device)
        sw = scaled_dot_product(q, k[:, lo:].unsqueeze(1), v[:, lo:].unsqueeze(1), mask=mask,
                                sink_logit=self.sink_logit, score_observer=self._observe,
                                logit_softcap=cfg.logit_softcap)
        g = torch.sigmoid(self.branch_gate(q))
        g = g / g.sum(-1, keepdim=True).clamp(min=1.0e-6)
        return self.output(g[..., 0:1] * comp + g[..., 1:2] * sel + g[..., 2:3] * sw)


__all__ = ["NSAttention", "block_compress", "selective_attention"]

"""Sliding-window MQA (first dense layers) and Heavily Compressed Attention (HCA).

SWA (reference ``core/attention/swa.py:27-138``): Q = q_norm(rope(q_up(q_compressor(h)))),
K = k_norm(rope(k_proj(h))) (RoPE *before* the norm), V = v_proj(h), one KV head,
causal window of ``sliding_window_size`` with a per-head sink.

HCA (reference ``core/attention/hca.py:31-169``): the SW branch of SWA plus dense
attention over k_norm'd compressed entries (K = V, compression m') that are complete
strictly before the query (``s*m' + m' - 1 < t``), *with* the sink; when there is no
sink, rows without any complete block are zeroed.  Output = out(compressed + sw).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from saint_llm_b200.config import AttentionConfig, HCAConfig
from saint_llm_b200.models.attention.common import scaled_dot_product
from saint_llm_b200.models.attention.csa import TokenLevelCompressor, _AttentionBase, _key_offset
from saint_llm_b200.models.linear import LinearFactory, default_linear
from saint_llm_b200.ops import backend


class SWAttention(_AttentionBase):
    def __init__(self, hidden_dim: int, attn: AttentionConfig, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__(hidden_dim, attn, linear_factory=linear_factory)
        self.k_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.v_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self._finish_init(hidden_dim, attn, linear_factory)

    def forward(self, h: Tensor, is_visual: Tensor | None = None, *,
                kv_cache: Any | None = None) -> Tensor:
        if kv_cache is None and backend.native_for(h):
            from saint_llm_b200.ops.attention import attention_forward

            return attention_forward(self, "swa", h, is_visual)
        off, cos, sin = self._positions(h, kv_cache)
        q = self._queries(h, cos, sin)
        k, v = self._sw_kv(h, cos, sin)
        if kv_cache is not None:
            k, v = kv_cache.append(k, v)
        return self.output(self._sw_branch(q, k, v, off, _key_offset(kv_cache)))


class HCA(_AttentionBase):
    def __init__(self, hidden_dim: int, attn: AttentionConfig, hca: HCAConfig, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__(hidden_dim, attn, linear_factory=linear_factory)
        self.hca_cfg = hca
        self.kv_compressor = TokenLevelCompressor(hidden_dim, attn.head_dim, hca.compression_rate,
                                                  linear_factory=linear_factory)
        self.k_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.v_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self._finish_init(hidden_dim, attn, linear_factory)

    def compressed_branch(self, q: Tensor, compressed: Tensor, q_start: int) -> Tensor:
        b, n_heads, t, d = q.shape
        n_blocks = compressed.shape[1]
        if n_blocks == 0:
            return q.new_zeros(b, n_heads, t, d)
        m = self.hca_cfg.compression_rate
        ck = self.k_norm(compressed).unsqueeze(1)
        qpos = torch.arange(q_start, q_start + t, device=q.device)[:, None]
        valid = torch.arange(n_blocks, device=q.device)[None, :] * m + (m - 1) < qpos
        out = scaled_dot_product(q, ck, ck, mask=valid, sink_logit=self.sink_logit)
        if self.sink_logit is None:
            out = torch.where(valid.any(-1)[None, None, :, None], out, torch.zeros_like(out))
        return out

    def forward(self, h: Tensor, is_visual: Tensor | None = None, *,
                kv_cache: Any | None = None) -> Tensor:
        if kv_cache is None and backend.native_for(h):
            from saint_llm_b200.ops.attention import attention_forward

            return attention_forward(self, "hca", h, is_visual)
        off, cos, sin = self._positions(h, kv_cache)
        q = self._queries(h, cos, sin)
        k, v = self._sw_kv(h, cos, sin)
        if kv_cache is not None:
            compressed, k, v = kv_cache.append(h, k, v, compressor=self.kv_compressor)
        else:
            compressed = self.kv_compressor(h)
        out = self.compressed_branch(q, compressed, off) + self._sw_branch(q, k, v, off, _key_offset(kv_cache))
        return self.output(out)


__all__ = ["HCA", "SWAttention"]

"""Compressed Sparse Attention (CSA) and its building blocks.

Reference behaviour (``core/attention/csa.py``):

* ``TokenLevelCompressor`` (``csa.py:41-88``) owns four H->c projections and two
  (m, c) positional biases, but only the *b* branch is consumed:
  ``compressed[s] = sum_j softmax_j(z_b[s*m+j] + bias_b[j]) * c_b[s*m+j]``; the
  trailing ``T mod m`` tokens are dropped.  The a-branch weights stay in the
  checkpoint (same key names) but never influence the output, so the fused path
  does not compute them.
* ``LightningIndexer`` (``csa.py:91-156``): ``score[t,s] = sum_h w[t,h] *
  relu(q[t,h] . k[s])`` (+0.5 * visual fraction of block s inside the relu'd head
  term), block s visible from t iff ``s*m + m - 1 < t`` (strict), top-k with
  invalid picks set to -1.  The indexer output is an integer selection, so no
  gradient reaches its parameters.
* ``CSA`` (``csa.py:192-375``): a top-k sparse branch over k_norm'd compressed
  entries (K = V, *no* sink, rows without a valid pick produce 0) plus a
  sliding-window branch (k_norm then RoPE on K, with sink); the two separately
  normalised outputs are summed before the grouped output projection.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import Tensor, nn

from saint_llm_b200.config import AttentionConfig, CSAConfig
from saint_llm_b200.models.attention.common import (
    RMSNorm,
    apply_partial_rope,
    rope_tables,
    scaled_dot_product,
    window_mask_at,
)
from saint_llm_b200.models.linear import LinearFactory, default_linear
from saint_llm_b200.ops import backend


def _key_offset(kv_cache: Any | None) -> int:
    """Global position of the first window key a cache returns (0: it returns all of them)."""
    return int(getattr(kv_cache, "key_offset", 0)) if kv_cache is not None else 0


class TokenLevelCompressor(nn.Module):
    def __init__(self, hidden_dim: int, c: int, m: int, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__()
        self.c = c
        self.m = m
        self.w_a_kv = linear_factory(hidden_dim, c, bias=False)
        self.w_b_kv = linear_factory(hidden_dim, c, bias=False)
        self.w_a_z = linear_factory(hidden_dim, c, bias=False)
        self.w_b_z = linear_factory(hidden_dim, c, bias=False)
        self.bias_a = nn.Parameter(torch.zeros(m, c))
        self.bias_b = nn.Parameter(torch.zeros(m, c))

    def pool(self, c_b: Tensor, z_b: Tensor) -> Tensor:
        """Softmax-pool (B, n*m, c) value/score projections into (B, n, c).  bf16 inputs on
        CUDA run the fused pooling kernel (fp32 math, one launch instead of ~25)."""
        if backend.native_for(c_b) and c_b.dtype == torch.bfloat16 and z_b.dtype == torch.bfloat16:
            from saint_llm_b200.ops.attention import _pool

            return _pool(c_b, z_b, self.bias_b, self.m).to(c_b.dtype)
        b, t, c = c_b.shape
        n = t // self.m
        z = z_b.reshape(b, n, self.m, c) + self.bias_b
        w = torch.softmax(z, dim=-2)
        return (w * c_b.reshape(b, n, self.m, c)).sum(dim=-2)

    def forward(self, h: Tensor) -> Tensor:
        b, t, _ = h.shape
        usable = (t // self.m) * self.m
        if usable == 0:
            return h.new_zeros(b, 0, self.c)
        hu = h[:, :usable]
        # The a-branch projections are part of the checkpoint but not of the output.
        return self.pool(self.w_b_kv(hu), self.w_b_z(hu))


class LightningIndexer(nn.Module):
    def __init__(self, hidden_dim: int, c_indexer: int, n_heads: int, top_k: int, m: int) -> None:
        super().__init__()
        self.c_indexer = c_indexer
        self.n_heads = n_heads
        self.top_k = top_k
        self.compressor = TokenLevelCompressor(hidden_dim, c_indexer, m)
        self.w_dq = nn.Linear(hidden_dim, c_indexer, bias=False)
        self.w_iuq = nn.Linear(c_indexer, n_heads * c_indexer, bias=False)
        self.w_w = nn.Linear(hidden_dim, n_heads, bias=False)

    def scores(self, h: Tensor, keys: Tensor, q_start: int, m: int,
               visual_bias: Tensor | None = None) -> Tensor:
        """(B, T, n_blocks) masked index scores for queries at absolute positions q_start.."""
        b, t, _ = h.shape
        n_blocks = keys.shape[1]
        q = self.w_iuq(self.w_dq(h)).view(b, t, self.n_heads, self.c_indexer)
        w = self.w_w(h)
        head = torch.einsum("bthc,bnc->bthn", q, keys).clamp(min=0.0)
        if visual_bias is not None:
            head = head + visual_bias[:, None, None, :] * 0.5
        s = (w.unsqueeze(-1) * head).sum(dim=-2)
        qpos = torch.arange(q_start, q_start + t, device=h.device)[:, None]
        block_end = torch.arange(n_blocks, device=h.device)[None, :] * m + (m - 1)
        return s.masked_fill(~(block_end < qpos), float("-inf"))

    @staticmethod
    def select(scores: Tensor, top_k: int) -> Tensor:
        b, t, n_blocks = scores.shape
        k = min(top_k, n_blocks)
        if k == 0:
            return torch.full((b, t, 0), -1, dtype=torch.long, device=scores.device)
        vals, idx = scores.topk(k, dim=-1)
        return torch.where(torch.isfinite(vals), idx, torch.full_like(idx, -1))

    def forward(self, h: Tensor, is_visual: Tensor | None = None) -> tuple[Tensor, Tensor]:
        b, t, _ = h.shape
        keys = self.compressor(h)
        n_blocks = keys.shape[1]
        if n_blocks == 0:
            return keys, torch.full((b, t, 0), -1, dtype=torch.long, device=h.device)
        # The reference derives the block length from T // n_blocks (equal to m
        # whenever m divides T) for both the visual bias and the causal mask.
        m_eff = t // n_blocks
        vis = None
        if is_visual is not None:
            vis = is_visual[:, : n_blocks * m_eff].reshape(b, n_blocks, m_eff).float().mean(-1)
        return keys, self.select(self.scores(h, keys, 0, m_eff, vis), self.top_k)


class GroupedOutputProjection(nn.Module):
    """Heads split into g groups; per-group linear to d_g; concat; final linear to D."""

    def __init__(self, hidden_dim: int, n_heads: int, head_dim: int, n_groups: int, d_g: int, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__()
        if n_heads % n_groups:
            raise ValueError("query_heads must be divisible by output_proj_groups")
        self.n_groups = n_groups
        self.heads_per_group = n_heads // n_groups
        self.d_g = d_g
        self.group_projs = nn.ModuleList(
            linear_factory(self.heads_per_group * head_dim, d_g, bias=False) for _ in range(n_groups)
        )
        self.final_proj = linear_factory(n_groups * d_g, hidden_dim, bias=False)

    def forward_flat(self, flat: Tensor) -> Tensor:
        """``flat`` is (..., H*head_dim) with heads contiguous."""
        parts = flat.chunk(self.n_groups, dim=-1)
        return self.final_proj(torch.cat([p(x) for p, x in zip(self.group_projs, parts, strict=True)], -1))

    def forward(self, attn_out: Tensor) -> Tensor:
        b, h, t, d = attn_out.shape
        return self.forward_flat(attn_out.transpose(1, 2).reshape(b, t, h * d))


class _AttentionBase(nn.Module):
    """Shared Q path, SW K/V path, sink, output projection and QK-Clip telemetry."""

    sw_norm_before_rope: bool = False

    def __init__(self, hidden_dim: int, attn: AttentionConfig, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.attn_cfg = attn
        self.q_compressor = linear_factory(hidden_dim, attn.query_compression_dim, bias=False)
        self.q_up = linear_factory(attn.query_compression_dim, attn.query_heads * attn.head_dim, bias=False)

    def _finish_init(self, hidden_dim: int, attn: AttentionConfig, linear_factory: LinearFactory) -> None:
        self.q_norm = RMSNorm(attn.head_dim)
        self.k_norm = RMSNorm(attn.head_dim)
        self.sink_logit: nn.Parameter | None = (
            nn.Parameter(torch.zeros(attn.query_heads)) if attn.use_attention_sink else None
        )
        self.output = GroupedOutputProjection(
            hidden_dim, attn.query_heads, attn.head_dim, attn.output_proj_groups,
            attn.attention_intermediate_dim, linear_factory=linear_factory,
        )
        # MuonClip telemetry: device-side max |QK^T/sqrt(d)| of the last forward
        # (the reference keeps a Python float and syncs the host every forward).
        self.register_buffer("max_attn_logit", torch.zeros(()), persistent=False)

    # ---- telemetry ---------------------------------------------------------------
    @property
    def _last_max_attn_logit(self) -> float:
        return float(self.max_attn_logit)

    @_last_max_attn_logit.setter
    def _last_max_attn_logit(self, value: float) -> None:
        self.max_attn_logit.fill_(float(value))

    def qk_clip_targets(self) -> list[Tensor]:
        return [self.q_up.weight, self.k_proj.weight]

    def _observe(self, scores: Tensor) -> None:
        self.max_attn_logit.copy_(scores.detach().abs().amax().to(self.max_attn_logit.dtype))

    # ---- shared pieces -----------------------------------------------------------
    def _queries(self, h: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
        b, t, _ = h.shape
        cfg = self.attn_cfg
        q = self.q_up(self.q_compressor(h)).view(b, t, cfg.query_heads, cfg.head_dim).transpose(1, 2)
        return self.q_norm(apply_partial_rope(q, cos, sin, cfg.rope_dim))

    def _sw_kv(self, h: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:
        rd = self.attn_cfg.rope_dim
        k = self.k_proj(h)
        if self.sw_norm_before_rope:
            k = apply_partial_rope(self.k_norm(k).unsqueeze(1), cos, sin, rd).squeeze(1)
        else:
            k = self.k_norm(apply_partial_rope(k, cos, sin, rd))
        return k, self.v_proj(h)

    def _sw_branch(self, q: Tensor, k: Tensor, v: Tensor, q_start: int, k_start: int = 0) -> Tensor:
        """Window branch for queries at global positions ``q_start..`` over keys at global
        positions ``k_start..`` (a cache may hold only the keys a window can reach)."""
        cfg = self.attn_cfg
        b, n_heads, t, d = q.shape
        # only the last `window` keys before the first query can be visible
        lo = max(0, q_start - cfg.sliding_window_size + 1 - k_start)
        k, v = k[:, lo:], v[:, lo:]
        mask = window_mask_at(q_start - k_start - lo, t, k.shape[1], cfg.sliding_window_size, q.device)
        return scaled_dot_product(
            q, k.unsqueeze(1), v.unsqueeze(1), mask=mask, sink_logit=self.sink_logit,
            score_observer=self._observe, logit_softcap=cfg.logit_softcap,
        )

    def _positions(self, h: Tensor, kv_cache: Any | None) -> tuple[int, Tensor, Tensor]:
        off = int(kv_cache.length) if kv_cache is not None else 0
        cos, sin = rope_tables(h.shape[1], self.attn_cfg.rope_dim, self.attn_cfg.rope_theta,
                               h.device, start=off)
        return off, cos, sin


class CSA(_AttentionBase):
    sw_norm_before_rope = True

    def __init__(self, hidden_dim: int, attn: AttentionConfig, csa: CSAConfig, *,
                 linear_factory: LinearFactory = default_linear) -> None:
        super().__init__(hidden_dim, attn, linear_factory=linear_factory)
        self.csa_cfg = csa
        self.kv_compressor = TokenLevelCompressor(hidden_dim, attn.head_dim, csa.compression_rate,
                                                  linear_factory=linear_factory)
        self.k_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.v_proj = linear_factory(hidden_dim, attn.head_dim, bias=False)
        self.indexer = LightningIndexer(hidden_dim, csa.indexer_head_dim, csa.indexer_query_heads,
                                        csa.attention_top_k, csa.compression_rate)
        self._finish_init(hidden_dim, attn, linear_factory)

    def sparse_branch(self, q: Tensor, compressed: Tensor, top_idx: Tensor) -> Tensor:
        """q (B,H,T,d); compressed (B,n,d) un-normalised; top_idx (B,T,k) with -1 = none."""
        b, n_heads, t, d = q.shape
        k_sel = top_idx.shape[-1]
        if compressed.shape[1] == 0 or k_sel == 0:
            return q.new_zeros(b, n_heads, t, d)
        valid = top_idx >= 0
        rows = torch.arange(b, device=q.device)[:, None, None]
        kv = self.k_norm(compressed[rows, top_idx.clamp(min=0)])  # (B,T,k,d), K = V
        s = torch.einsum("bhtd,btkd->bthk", q, kv) / math.sqrt(d)
        s = s.masked_fill(~valid[:, :, None, :], float("-inf"))
        has_any = valid.any(-1)[:, :, None, None]
        s = torch.where(has_any, s, torch.zeros_like(s))
        p = torch.softmax(s, dim=-1)
        out = torch.einsum("bthk,btkd->bthd", p, kv)
        out = torch.where(has_any, out, torch.zeros_like(out))
        return out.transpose(1, 2)

    def forward(self, h: Tensor, is_visual: Tensor | None = None, *,
                kv_cache: Any | None = None) -> Tensor:
        if kv_cache is None and backend.native_for(h):
            from saint_llm_b200.ops.attention import attention_forward

            return attention_forward(self, "csa", h, is_visual)
        off, cos, sin = self._positions(h, kv_cache)
        q = self._queries(h, cos, sin)
        k_new, v_new = self._sw_kv(h, cos, sin)
        m = self.csa_cfg.compression_rate
        if kv_cache is not None and is_visual is not None and getattr(kv_cache, "carries_visual_bias", False):
            # a context-parallel view: the sequence is whole, only sharded, so the indexer keeps
            # the visual cohesion bias of its blocks (gathered with the compressed entries)
            compressed, idx_keys, k, v, vis_bias = kv_cache.append(
                h, k_new, v_new, compressor=self.kv_compressor,
                indexer_compressor=self.indexer.compressor, is_visual=is_visual,
            )
            top_idx = self.indexer.select(self.indexer.scores(h, idx_keys, off, m, vis_bias), self.indexer.top_k)
        elif kv_cache is not None:
            # a decode cache: like the reference, the cached path has no visual bias
            compressed, idx_keys, k, v = kv_cache.append(
                h, k_new, v_new, compressor=self.kv_compressor,
                indexer_compressor=self.indexer.compressor,
            )
            top_idx = self.topk_cached(h, idx_keys, off, m)
        else:
            _, top_idx = self.indexer(h, is_visual=is_visual)
            compressed = self.kv_compressor(h)
            k, v = k_new, v_new
        out = self.sparse_branch(q, compressed, top_idx) + self._sw_branch(q, k, v, off, _key_offset(kv_cache))
        return self.output(out)

    def topk_cached(self, h: Tensor, idx_keys: Tensor, q_start: int, m: int) -> Tensor:
        """Indexer selection against cached compressed keys (absolute positions)."""
        n_blocks = idx_keys.shape[1]
        if n_blocks == 0:
            return torch.full((h.shape[0], h.shape[1], 0), -1, dtype=torch.long, device=h.device)
        return self.indexer.select(self.indexer.scores(h, idx_keys, q_start, m), self.indexer.top_k)

    # reference-compatible private name
    def _indexer_topk_cached(self, h: Tensor, k_indexer_comp: Tensor, *, cache_offset: int,
                             total_len: int, n_blocks: int, m: int,
                             is_visual: Tensor | None = None) -> Tensor:
        del total_len, n_blocks, is_visual
        return self.topk_cached(h, k_indexer_comp, cache_offset, m)


__all__ = ["CSA", "GroupedOutputProjection", "LightningIndexer", "TokenLevelCompressor"]

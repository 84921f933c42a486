"""Multi-token prediction heads (reference ``core/mtp.py:16-62``).

Depth k (0-based) combines ``RMSNorm(h_k)`` with ``RMSNorm(embedding shifted left by
k+1)`` (zero-padded at the end) through one ``2D -> D`` linear, chained from the
final hidden state; logits come from the tied LM head.  There is no transformer
block inside an MTP module.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from saint_llm_b200.config import MTPConfig
from saint_llm_b200.models.attention.common import RMSNorm
from saint_llm_b200.models.linear import Linear


class MTPModule(nn.Module):
    def __init__(self, hidden_dim: int, vocab_size: int, rms_norm_eps: float = 1.0e-6) -> None:
        super().__init__()
        del vocab_size
        self.norm_h = RMSNorm(hidden_dim, eps=rms_norm_eps)
        self.norm_e = RMSNorm(hidden_dim, eps=rms_norm_eps)
        self.combine = Linear(2 * hidden_dim, hidden_dim, bias=False)

    def forward(self, hidden: Tensor, prev_token_embed: Tensor) -> Tensor:
        return self.combine(torch.cat([self.norm_h(hidden), self.norm_e(prev_token_embed)], dim=-1))


def shift_left(x: Tensor, shift: int) -> Tensor:
    """x[:, shift:] padded with zeros at the end (all zeros when T <= shift)."""
    if x.shape[1] <= shift:
        return torch.zeros_like(x)
    return torch.cat([x[:, shift:], x.new_zeros(x.shape[0], shift, x.shape[-1])], dim=1)


class MTPStack(nn.Module):
    def __init__(self, hidden_dim: int, vocab_size: int, cfg: MTPConfig, rms_norm_eps: float = 1.0e-6) -> None:
        super().__init__()
        self.depth = cfg.depth
        self.modules_ = nn.ModuleList(MTPModule(hidden_dim, vocab_size, rms_norm_eps) for _ in range(cfg.depth))

    def forward(self, hidden: Tensor, embeddings: Tensor) -> list[Tensor]:
        outs: list[Tensor] = []
        cur = hidden
        for k, mod in enumerate(self.modules_):
            cur = mod(cur, shift_left(embeddings, k + 1))
            outs.append(cur)
        return outs


__all__ = ["MTPModule", "MTPStack", "shift_left"]

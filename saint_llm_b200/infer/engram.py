"""Engram conditional memory: an N-gram-hashed embedding table added to the residual
stream through a zero-initialised projection (reference: ``saint_llm_inference/engram.py``).

The reference hashes each position's trailing N-gram with SHA1 in a Python loop.  Here the
bucket ids of all positions come from one vectorised rolling hash over the token tensor
(int64 multiply-xorshift, on whatever device the ids live), the table stays in host
memory (pinned when CUDA is present) and only the gathered rows cross to the GPU.  Bucket
ids therefore differ from the reference's SHA1 buckets; tables are not interchangeable.
"""

from __future__ import annotations

import torch
from pydantic import BaseModel, ConfigDict
from torch import Tensor, nn

_M1 = 0x9E3779B97F4A7C15 - (1 << 64)   # golden-ratio odd constant as signed int64
_M2 = 0xBF58476D1CE4E5B9 - (1 << 64)


class EngramConfig(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")
    n_gram: int = 4
    n_buckets: int = 65_536
    embedding_dim: int = 128
    enabled: bool = False


def _mix(x: Tensor) -> Tensor:
    x = x ^ (x >> 31)
    x = x * _M2
    return x ^ (x >> 29)


def ngram_buckets(ids: Tensor, n_gram: int, n_buckets: int) -> Tensor:
    """Bucket id of the trailing ``n_gram``-gram ending at every position of ``ids`` (..., T).
    Positions with fewer than ``n_gram`` predecessors hash the shorter prefix."""
    x = ids.to(torch.int64)
    h = torch.zeros_like(x)
    for j in range(n_gram):
        shifted = torch.nn.functional.pad(x, (j, 0), value=-1)[..., :x.shape[-1]] if j else x
        valid = shifted >= 0
        h = torch.where(valid, _mix(h * _M1 + shifted + 1), h)
    return torch.remainder(h, n_buckets)


def trailing_bucket(recent_token_ids: list[int], n_gram: int, n_buckets: int) -> int:
    return int(ngram_buckets(torch.tensor([recent_token_ids[-n_gram:]]), n_gram, n_buckets)[0, -1])


class EngramTable(nn.Module):
    def __init__(self, cfg: EngramConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.register_buffer("embeddings", torch.zeros(cfg.n_buckets, cfg.embedding_dim), persistent=True)

    def _apply(self, fn, recurse=True):  # noqa: ANN001 - keep the table in host memory on .to(cuda)
        return self

    def pin(self) -> EngramTable:
        if torch.cuda.is_available() and not self.embeddings.is_pinned():
            self.embeddings = self.embeddings.pin_memory()
        return self

    def lookup(self, recent_token_ids: list[int]) -> Tensor:
        if not recent_token_ids:
            return torch.zeros(self.cfg.embedding_dim)
        return self.embeddings[trailing_bucket(recent_token_ids, self.cfg.n_gram, self.cfg.n_buckets)]

    def lookup_batch(self, ids: Tensor) -> Tensor:
        """(B, T) ids -> (B, T, E) rows (host tensor)."""
        b = ngram_buckets(ids.cpu(), self.cfg.n_gram, self.cfg.n_buckets)
        return self.embeddings[b]

    @torch.no_grad()
    def update(self, recent_token_ids: list[int], delta: Tensor) -> None:
        if recent_token_ids:
            self.embeddings[trailing_bucket(recent_token_ids, self.cfg.n_gram, self.cfg.n_buckets)] += delta.cpu()


class EngramHook(nn.Module):
    """``hidden + proj(table[ngram(ids)])``; identity while disabled or untrained."""

    def __init__(self, hidden_dim: int, table: EngramTable) -> None:
        super().__init__()
        self.table = table
        self.proj = nn.Linear(table.cfg.embedding_dim, hidden_dim, bias=False)
        nn.init.zeros_(self.proj.weight)

    def forward(self, hidden: Tensor, recent_token_ids: Tensor) -> Tensor:
        if not self.table.cfg.enabled:
            return hidden
        if hidden.dim() != 3:
            raise ValueError(f"hidden must be (B,T,D); got {tuple(hidden.shape)}")
        rows = self.table.lookup_batch(recent_token_ids)
        rows = rows.to(hidden.device, non_blocking=True).to(self.proj.weight.dtype)
        return hidden + self.proj(rows).to(hidden.dtype)


__all__ = ["EngramConfig", "EngramHook", "EngramTable", "ngram_buckets"]

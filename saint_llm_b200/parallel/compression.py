"""Gradient compression for bandwidth-limited synchronisation
(reference: ``saint_llm_distributed/gradient_compression.py:33-271``): top-k by magnitude,
top-k with error feedback, decompression, and SparseLoCo -- top-k that skips coordinates a
peer already sent, tracked with a Bloom filter that peers OR-merge.

The Bloom filter here hashes all candidate indices at once on the tensor's device
(``k`` multiply-xorshift hashes of the int64 index), so a filter query or insert is a
vectorised gather/scatter instead of a per-index Python loop.  Bit positions therefore
differ from the reference's SHA1 hashing; filters are exchanged between peers of this
implementation only.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
from torch import Tensor


@dataclass(frozen=True)
class CompressedGradient:
    indices: Tensor
    values: Tensor
    shape: tuple[int, ...]
    n_total: int

    def density(self) -> float:
        return 0.0 if self.n_total == 0 else self.indices.numel() / self.n_total


def _k_for(n: int, density: float) -> int:
    if not 0.0 < density <= 1.0:
        raise ValueError(f"density must be in (0, 1]; got {density}")
    return max(1, round(density * n))


def top_k_compression(grad: Tensor, *, density: float) -> CompressedGradient:
    flat = grad.reshape(-1)
    k = min(_k_for(flat.numel(), density), flat.numel())
    idx = flat.abs().topk(k, sorted=False).indices
    return CompressedGradient(idx, flat[idx], tuple(grad.shape), flat.numel())


@dataclass
class TopKWithResidualCompressor:
    """Error feedback: what is not sent this step is added to the next step's gradient."""

    density: float
    _residual: Tensor | None = field(default=None, init=False, repr=False)

    def step(self, grad: Tensor) -> CompressedGradient:
        if self._residual is None or self._residual.shape != grad.shape:
            self._residual = torch.zeros_like(grad)
        adj = grad + self._residual
        c = top_k_compression(adj, density=self.density)
        self._residual = adj.clone()
        self._residual.view(-1)[c.indices] = 0
        return c

    def reset(self) -> None:
        self._residual = None


def decompress(c: CompressedGradient, *, dtype: torch.dtype | None = None) -> Tensor:
    out = torch.zeros(c.n_total, dtype=dtype or c.values.dtype, device=c.values.device)
    out[c.indices] = c.values.to(out.dtype)
    return out.reshape(c.shape)


_M1 = 0x9E3779B97F4A7C15 - (1 << 64)
_M2 = 0xBF58476D1CE4E5B9 - (1 << 64)


def _bloom_positions(idx: Tensor, n_hashes: int, m_bits: int) -> Tensor:
    """(n, n_hashes) bit positions for int64 indices."""
    x = idx.to(torch.int64).unsqueeze(-1) * _M1 + torch.arange(1, n_hashes + 1, device=idx.device) * _M2
    x = x ^ (x >> 31)
    x = x * _M2
    x = x ^ (x >> 29)
    return torch.remainder(x, m_bits)


def bloom_size_for(n_items: int, false_pos_rate: float = 0.01) -> tuple[int, int]:
    """Standard sizing: m = -n ln p / ln^2 2 bits, k = (m / n) ln 2 hashes."""
    m = max(64, int(-n_items * math.log(false_pos_rate) / math.log(2) ** 2))
    return m, max(1, round(m / max(n_items, 1) * math.log(2)))


@dataclass(frozen=True)
class SparseLoCoBloom:
    bits: Tensor  # bool, length m_bits
    m_bits: int
    n_hashes: int

    @classmethod
    def empty(cls, *, m_bits: int, n_hashes: int, device: torch.device | str | None = None) -> SparseLoCoBloom:
        return cls(torch.zeros(m_bits, dtype=torch.bool, device=device), m_bits, n_hashes)

    def contains_many(self, idx: Tensor) -> Tensor:
        return self.bits[_bloom_positions(idx.to(self.bits.device), self.n_hashes, self.m_bits)].all(-1)

    def contains(self, idx: int) -> bool:
        return bool(self.contains_many(torch.tensor([idx]))[0])

    def add_many(self, idx: Tensor) -> None:
        self.bits[_bloom_positions(idx.to(self.bits.device), self.n_hashes, self.m_bits).reshape(-1)] = True

    def add(self, idx: int) -> None:
        self.add_many(torch.tensor([idx]))

    def merged_with(self, other: SparseLoCoBloom) -> SparseLoCoBloom:
        if (self.m_bits, self.n_hashes) != (other.m_bits, other.n_hashes):
            raise ValueError("bloom filters must share m_bits and n_hashes to merge")
        return SparseLoCoBloom(self.bits | other.bits.to(self.bits.device), self.m_bits, self.n_hashes)


def sparse_loco_compress(grad: Tensor, *, density: float, peer_bloom: SparseLoCoBloom | None = None,
                         bloom_false_pos_rate: float = 0.01) -> tuple[CompressedGradient, SparseLoCoBloom]:
    """Top-k over the local pseudo-gradient skipping indices in ``peer_bloom``; returns the
    compressed gradient and a fresh filter of the indices sent (sized for k)."""
    flat = grad.reshape(-1)
    n = flat.numel()
    k = _k_for(n, density)
    cand = flat.abs().topk(min(n, max(2 * k, 64)), sorted=True).indices
    m, h = bloom_size_for(k, bloom_false_pos_rate) if peer_bloom is None else (peer_bloom.m_bits, peer_bloom.n_hashes)
    if peer_bloom is not None:
        fresh = cand[~peer_bloom.contains_many(cand)]
        cand = fresh if fresh.numel() else cand[:1]
    kept = cand[:k]
    out = SparseLoCoBloom.empty(m_bits=m, n_hashes=h, device=grad.device)
    out.add_many(kept)
    return CompressedGradient(kept, flat[kept], tuple(grad.shape), n), out


__all__ = ["CompressedGradient", "SparseLoCoBloom", "TopKWithResidualCompressor", "bloom_size_for", "decompress",
           "sparse_loco_compress", "top_k_compression"]

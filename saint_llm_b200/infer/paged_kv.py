"""Paged KV storage for serving many sequences of different lengths from one pool.

The static decoder keeps fixed per-layer buffers sized for the longest sequence; a server
with requests of mixed lengths wastes most of that.  Here every cache stream (window K / V,
compressed entries, indexer keys -- any (rows, dim) tensor that grows with the sequence)
lives in fixed-size pages of a shared pool, and each sequence owns a block table: the list
of its pages in order.  Pages are allocated when a stream crosses a page boundary and
returned when the request finishes, so memory follows the live tokens.

* ``PagePool``: the storage (n_pages, page_rows, dim) and a free list (host side).
* ``PagedStream``: one sequence's stream -- block table, length, append, gather.
* ``PagedKVManager``: per-request streams for every (layer, stream name); admit / append /
  release; batched block tables and padded gathers for a set of requests.
* ``paged_attention``: the attention oracle over paged keys / values (block tables +
  lengths), equal to attention over the contiguous rows.

(The reference's caches are per-sequence preallocated tensors, ``inference/kv_cache.py:32-427``;
paging is this framework's addition for config 5's serving setting.)
"""

from __future__ import annotations

import math
from collections.abc import Iterable

import torch
from torch import Tensor


class PoolExhausted(RuntimeError):
    """No free page left in the pool."""


class PagePool:
    def __init__(self, n_pages: int, page_rows: int, dim: int, *, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None) -> None:
        if n_pages <= 0 or page_rows <= 0:
            raise ValueError("n_pages and page_rows must be positive")
        self.page_rows, self.dim = page_rows, dim
        self.storage = torch.zeros(n_pages, page_rows, dim, dtype=dtype, device=device)
        self._free = list(range(n_pages - 1, -1, -1))  # pop() hands out low page ids first
        self._is_free = set(self._free)

    @property
    def n_pages(self) -> int:
        return self.storage.shape[0]

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def alloc(self) -> int:
        if not self._free:
            raise PoolExhausted(f"all {self.n_pages} pages are in use")
        p = self._free.pop()
        self._is_free.discard(p)
        return p

    def alloc_many(self, n: int) -> list[int]:
        """``n`` pages at once, or none (PoolExhausted) when fewer are free."""
        if n > len(self._free):
            raise PoolExhausted(f"{n} pages requested, {len(self._free)} of {self.n_pages} free")
        return [self.alloc() for _ in range(n)]

    def free(self, pages: Iterable[int]) -> None:
        """Return pages to the pool.  A page that is already free (a double free would hand
        one page to two requests) or not a page of this pool raises, and nothing is freed."""
        pages = list(pages)
        bad = [p for p in pages if not 0 <= p < self.n_pages or p in self._is_free]
        if bad or len(set(pages)) != len(pages):
            raise ValueError(f"pages already free, repeated or out of range: {sorted(set(bad)) or pages}")
        for p in pages:
            self._free.append(p)
            self._is_free.add(p)


class PagedStream:
    """One sequence's rows in ``pool`` pages."""

    def __init__(self, pool: PagePool) -> None:
        self.pool = pool
        self.pages: list[int] = []
        self.length = 0

    def append(self, rows: Tensor) -> None:
        """rows (n, dim).  All or nothing: the pages the rows need are reserved before any
        row is written, so a full pool raises PoolExhausted with the stream unchanged."""
        if rows.dim() != 2 or rows.shape[1] != self.pool.dim:
            raise ValueError(f"rows must be (n, {self.pool.dim})")
        pr = self.pool.page_rows
        n = rows.shape[0]
        need = math.ceil((self.length + n) / pr) - len(self.pages)
        fresh = self.pool.alloc_many(max(need, 0))
        self.pages.extend(fresh)
        i = 0
        while i < n:
            off = self.length % pr
            take = min(pr - off, n - i)
            self.pool.storage[self.pages[self.length // pr], off:off + take] = rows[i:i + take].to(
                self.pool.storage.dtype)
            self.length += take
            i += take

    def gather(self) -> Tensor:
        if self.length == 0:
            return self.pool.storage.new_zeros(0, self.pool.dim)
        idx = torch.tensor(self.pages, device=self.pool.storage.device)
        return self.pool.storage.index_select(0, idx).reshape(-1, self.pool.dim)[:self.length]

    def truncate(self, length: int) -> None:
        """Keep the first ``length`` rows (speculative-decoding rollback); frees whole pages."""
        if not 0 <= length <= self.length:
            raise ValueError("truncate length out of range")
        keep = math.ceil(length / self.pool.page_rows)
        self.pool.free(self.pages[keep:])
        self.pages = self.pages[:keep]
        self.length = length

    def release(self) -> None:
        self.pool.free(self.pages)
        self.pages, self.length = [], 0


class PagedKVManager:
    """Streams of every admitted request, one pool per stream name (pools of one name share a
    row width, e.g. ``"k"`` / ``"v"`` of head_dim, ``"entries"`` of the compressed width)."""

    def __init__(self, pools: dict[str, PagePool], n_layers: int) -> None:
        self.pools, self.n_layers = pools, n_layers
        self.streams: dict[object, dict[tuple[int, str], PagedStream]] = {}

    def admit(self, req: object) -> None:
        if req in self.streams:
            raise KeyError(f"request {req!r} already admitted")
        self.streams[req] = {(layer, name): PagedStream(pool) for layer in range(self.n_layers)
                             for name, pool in self.pools.items()}

    def append(self, req: object, layer: int, name: str, rows: Tensor) -> None:
        self.streams[req][(layer, name)].append(rows)

    def length(self, req: object, layer: int, name: str) -> int:
        return self.streams[req][(layer, name)].length

    def release(self, req: object) -> None:
        for s in self.streams.pop(req).values():
            s.release()

    def block_tables(self, reqs: list[object], layer: int, name: str) -> tuple[Tensor, Tensor]:
        """(B, max_pages) int32 page ids (-1 padded) and (B,) int32 lengths."""
        ss = [self.streams[r][(layer, name)] for r in reqs]
        width = max((len(s.pages) for s in ss), default=0)
        dev = self.pools[name].storage.device
        table = torch.full((len(ss), max(width, 1)), -1, dtype=torch.int32)
        for i, s in enumerate(ss):
            if s.pages:
                table[i, :len(s.pages)] = torch.tensor(s.pages, dtype=torch.int32)
        lengths = torch.tensor([s.length for s in ss], dtype=torch.int32)
        return table.to(dev), lengths.to(dev)

    def gather_padded(self, reqs: list[object], layer: int, name: str) -> tuple[Tensor, Tensor]:
        """(B, max_len, dim) rows (zero padded) and (B,) lengths."""
        rows = [self.streams[r][(layer, name)].gather() for r in reqs]
        pool = self.pools[name]
        out = pool.storage.new_zeros(len(rows), max((x.shape[0] for x in rows), default=0), pool.dim)
        for i, x in enumerate(rows):
            out[i, :x.shape[0]] = x
        return out, torch.tensor([x.shape[0] for x in rows], dtype=torch.int32, device=out.device)


def paged_attention(q: Tensor, k_pool: PagePool, v_pool: PagePool, block_table: Tensor, lengths: Tensor, *,
                    sink: Tensor | None = None) -> Tensor:
    """Single-token attention over paged K / V: q (B, H, d); block_table (B, P) int32 (-1 =
    none); lengths (B,).  MQA (one K/V head).  Returns (B, H, d) in fp32."""
    b, h, d = q.shape
    tbl = block_table.long().clamp(min=0)
    k = k_pool.storage[tbl].reshape(b, -1, d).float()      # (B, P * page_rows, d)
    v = v_pool.storage[tbl].reshape(b, -1, d).float()
    pos = torch.arange(k.shape[1], device=q.device)
    valid = pos[None, :] < lengths.long()[:, None]
    s = torch.einsum("bhd,bnd->bhn", q.float(), k) / math.sqrt(d)
    s = s.masked_fill(~valid[:, None, :], float("-inf"))
    if sink is not None:
        s = torch.cat([s, sink.float().view(1, h, 1).expand(b, h, 1)], dim=-1)
    p = torch.softmax(s, dim=-1)
    if sink is not None:
        p = p[..., :-1]
    return torch.einsum("bhn,bnd->bhd", p, v)


__all__ = ["PagePool", "PagedKVManager", "PagedStream", "PoolExhausted", "paged_attention"]

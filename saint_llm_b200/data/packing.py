"""Concat-and-chunk packing of tokenised documents into fixed ``(B, T)`` windows.

Same contract as the reference's ``saint_llm_data/packing.py:23-137``: an EOS after every
document, ``segment_ids`` numbering documents in stream order, optional right padding of
the residual window (segment id of the last document) and, for batches, padding rows
with segment id ``-1``.  The bulk path (:func:`pack_flat`) runs in the native extension
over one flat token array instead of per-token Python lists.
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator
from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass(frozen=True)
class PackedBatch:
    tokens: Tensor
    segment_ids: Tensor

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.tokens.shape)


class _Packer:
    """Streaming state: a ring of pending tokens/segments kept as tensors, not lists."""

    def __init__(self, seq_len: int, eos: int) -> None:
        if seq_len <= 0:
            raise ValueError(f"seq_len must be positive; got {seq_len}")
        self.seq_len, self.eos = seq_len, eos
        self.tok: list[Tensor] = []
        self.seg: list[Tensor] = []
        self.n = 0
        self.next_seg = 0

    def push(self, doc: list[int] | Tensor) -> None:
        d = torch.as_tensor(doc, dtype=torch.long).reshape(-1)
        if d.numel() == 0:
            return
        self.tok.append(torch.cat([d, d.new_tensor([self.eos])]))
        self.seg.append(torch.full((d.numel() + 1,), self.next_seg, dtype=torch.long))
        self.next_seg += 1
        self.n += d.numel() + 1

    def windows(self) -> Iterator[tuple[Tensor, Tensor]]:
        if self.n < self.seq_len:
            return
        tok, seg = torch.cat(self.tok), torch.cat(self.seg)
        full = (self.n // self.seq_len) * self.seq_len
        for s in range(0, full, self.seq_len):
            yield tok[s:s + self.seq_len], seg[s:s + self.seq_len]
        self.tok, self.seg = [tok[full:]], [seg[full:]]
        self.n -= full

    def residual(self, pad: int) -> tuple[Tensor, Tensor] | None:
        if self.n == 0:
            return None
        tok, seg = torch.cat(self.tok), torch.cat(self.seg)
        k = self.seq_len - self.n
        return (torch.cat([tok, tok.new_full((k,), pad)]),
                torch.cat([seg, seg.new_full((k,), int(seg[-1]))]))


def pack_sequences(docs: Iterable[list[int]], *, seq_len: int, eos_token_id: int, pad_token_id: int = 0,
                   drop_last: bool = True) -> Iterator[PackedBatch]:
    """Yield ``(1, seq_len)`` windows from a stream of documents."""
    p = _Packer(seq_len, eos_token_id)
    for doc in docs:
        p.push(doc)
        for t, s in p.windows():
            yield PackedBatch(t.unsqueeze(0), s.unsqueeze(0))
    if not drop_last:
        r = p.residual(pad_token_id)
        if r is not None:
            yield PackedBatch(r[0].unsqueeze(0), r[1].unsqueeze(0))


def pack_into_batch(docs: Iterable[list[int]], *, batch_size: int, seq_len: int, eos_token_id: int,
                    pad_token_id: int = 0, drop_last: bool = True) -> Iterator[PackedBatch]:
    """Group packed windows into ``(batch_size, seq_len)`` batches."""
    rows: list[PackedBatch] = []
    for w in pack_sequences(docs, seq_len=seq_len, eos_token_id=eos_token_id, pad_token_id=pad_token_id,
                            drop_last=drop_last):
        rows.append(w)
        if len(rows) == batch_size:
            yield PackedBatch(torch.cat([r.tokens for r in rows]), torch.cat([r.segment_ids for r in rows]))
            rows = []
    if rows and not drop_last:
        k = batch_size - len(rows)
        tok = torch.cat([r.tokens for r in rows] + [torch.full((k, seq_len), pad_token_id, dtype=torch.long)])
        seg = torch.cat([r.segment_ids for r in rows] + [torch.full((k, seq_len), -1, dtype=torch.long)])
        yield PackedBatch(tok, seg)


def pack_flat(tokens: Tensor, doc_offsets: Tensor, *, seq_len: int, eos_token_id: int, pad_token_id: int = 0,
              drop_last: bool = True) -> PackedBatch:
    """Pack a whole corpus at once: ``tokens`` is the concatenation of all documents and
    ``doc_offsets`` (n_docs + 1) their boundaries.  Runs in the native extension."""
    from saint_llm_b200.ops.backend import ext

    t, s = ext().pack_documents(tokens.to(torch.int64).contiguous(), doc_offsets.to(torch.int64).contiguous(),
                                int(seq_len), int(eos_token_id), int(pad_token_id), bool(drop_last))
    return PackedBatch(t, s)


__all__ = ["PackedBatch", "pack_flat", "pack_into_batch", "pack_sequences"]

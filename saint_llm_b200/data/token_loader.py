"""Pretraining input pipeline: binary token shards, read by a native background loader
into pinned host buffers and copied to the GPU on a side stream.

The reference streams text through tokenisation and Python packing on every step
(``saint_llm_data/dataset.py:59-115``); at B200 step rates that host work is the
bottleneck, so pretraining here reads pre-tokenised shards.  :func:`write_token_shard`
writes the shard format; :class:`ShardedTokenLoader` yields device batches.
"""

from __future__ import annotations

import struct
from collections.abc import Iterator, Sequence
from pathlib import Path

import numpy as np
import torch
from torch import Tensor

_MAGIC = b"SV4TOKS\0"


def write_token_shard(path: str | Path, tokens: Sequence[int] | np.ndarray | Tensor, *, vocab_size: int) -> Path:
    """Write ``tokens`` as a shard (uint16 when the vocabulary fits, else uint32)."""
    arr = tokens.cpu().numpy() if isinstance(tokens, Tensor) else np.asarray(tokens)
    dtype = np.uint16 if vocab_size <= 65536 else np.uint32
    if arr.size and (arr.min() < 0 or arr.max() >= vocab_size):
        raise ValueError("token id outside [0, vocab_size)")
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("wb") as f:
        f.write(_MAGIC + struct.pack("<IIQQ", 1, np.dtype(dtype).itemsize, arr.size, 0))
        f.write(arr.astype(dtype, copy=False).tobytes())
    return path


def read_token_shard(path: str | Path) -> np.ndarray:
    raw = Path(path).read_bytes()
    if raw[:8] != _MAGIC:
        raise ValueError(f"{path} is not a token shard")
    _, width, n, _ = struct.unpack("<IIQQ", raw[8:32])
    return np.frombuffer(raw[32:32 + n * width], dtype=np.uint16 if width == 2 else np.uint32)


class ShardedTokenLoader:
    """Random ``(batch, seq_len)`` windows from token shards, prefetched by a native thread.

    Windows are a deterministic function of ``(seed, rank, step, row)``, so a resumed run
    (``skip(step)``) and every data-parallel rank draw disjoint, reproducible samples.
    Iterating yields int64 tensors on ``device``; the host-to-device copy of batch i+1
    runs on a side stream while step i computes.
    """

    def __init__(self, paths: Sequence[str | Path], *, batch_size: int, seq_len: int, seed: int = 0,
                 rank: int = 0, world_size: int = 1, prefetch: int = 4, device: torch.device | str | None = None):
        from saint_llm_b200.ops.backend import ext

        self.device = torch.device(device) if device is not None else torch.device("cpu")
        pin = self.device.type == "cuda"
        self._impl = ext().TokenShardLoader([str(p) for p in paths], batch_size, seq_len, seed, rank, world_size,
                                            max(2, prefetch), pin)
        self._pending: tuple[int, torch.cuda.Event | None] | None = None
        self._stream = torch.cuda.Stream(self.device) if pin else None
        self.h2d_bytes = batch_size * seq_len * 8

    @property
    def total_windows(self) -> int:
        return int(self._impl.total_windows)

    def _retire(self) -> None:
        if self._pending is not None:
            slot, ev = self._pending
            if ev is not None:
                ev.synchronize()
            self._impl.release(slot)
            self._pending = None

    def next(self) -> Tensor:
        self._retire()
        slot, host = self._impl.next()
        if self._stream is None:
            out = host.clone()
            self._impl.release(slot)
            return out
        with torch.cuda.stream(self._stream):
            out = host.to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._stream)
        torch.cuda.current_stream(self.device).wait_stream(self._stream)
        out.record_stream(torch.cuda.current_stream(self.device))
        self._pending = (slot, ev)
        return out

    def __iter__(self) -> Iterator[Tensor]:
        while True:
            yield self.next()

    def close(self) -> None:
        self._retire()
        self._impl.close()

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


__all__ = ["ShardedTokenLoader", "read_token_shard", "write_token_shard"]

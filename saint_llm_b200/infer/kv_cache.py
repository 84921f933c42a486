"""Heterogeneous KV cache for SWA / HCA / CSA attention layers.

Contract (same as the reference's ``saint_llm_inference/kv_cache.py:32-427``, which the
attention modules call through duck typing):

* every layer keeps post-RoPE sliding-window K/V for the whole history and a ``length``;
* HCA and CSA layers also keep compressed blocks: raw hidden states of the unfinished
  block wait in an ``h``-buffer and are compressed, by the layer's own compressor, as
  soon as ``compression_rate`` of them are present (CSA runs its indexer compressor in
  lock step);
* ``append`` returns views of everything cached so far.

Here one class, :class:`CompressedKVLayer`, implements the compressed streams for any
number of compressors (HCA: 1, CSA: 2) on top of the window cache, and every buffer is
allocated once at its maximum size so the decode loop never reallocates.  ``truncate``
rolls a layer back to an earlier length (speculative decoding).  Rolling back across an
emitted compressed block needs that block's raw hidden states again, so a layer built
with ``keep_history=True`` keeps the raw hidden states of the whole history; otherwise
only the unfinished block is kept (``(B, m, hidden)``) and such a rollback raises.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor


def _check3(*ts: Tensor) -> None:
    for t in ts:
        if t.dim() != 3:
            raise ValueError(f"cache inputs must be (B, T, *); got {tuple(t.shape)}")


class SWAKVCacheLayer:
    """Append-only window K/V (``(B, max_seq_len, head_dim)`` each)."""

    def __init__(self, max_seq_len: int, head_dim: int, *, batch_size: int = 1,
                 device: torch.device | str | None = None, dtype: torch.dtype = torch.float32) -> None:
        if max_seq_len <= 0:
            raise ValueError(f"max_seq_len must be positive; got {max_seq_len}")
        self.max_seq_len, self.head_dim, self.batch_size = max_seq_len, head_dim, batch_size
        self.k = torch.zeros(batch_size, max_seq_len, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.length = 0

    def _reserve(self, n: int) -> int:
        if self.length + n > self.max_seq_len:
            raise RuntimeError(f"{type(self).__name__} overflow: appending {n} tokens at length {self.length} "
                               f"exceeds max_seq_len={self.max_seq_len}")
        return self.length

    def _write_window(self, k_new: Tensor, v_new: Tensor) -> None:
        s = self._reserve(k_new.shape[1])
        self.k[:, s:s + k_new.shape[1]] = k_new
        self.v[:, s:s + v_new.shape[1]] = v_new

    def append(self, k_new: Tensor, v_new: Tensor) -> tuple[Tensor, Tensor]:
        _check3(k_new, v_new)
        self._write_window(k_new, v_new)
        self.length += k_new.shape[1]
        return self.k[:, :self.length], self.v[:, :self.length]

    # reference attribute names for the window buffers of compressed layers
    @property
    def sw_k(self) -> Tensor:
        return self.k

    @property
    def sw_v(self) -> Tensor:
        return self.v

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate length {self.length} to {length}")
        self.length = length

    def reset(self) -> None:
        self.length = 0

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self._buffers())

    def _buffers(self) -> list[Tensor]:
        return [self.k, self.v]


class CompressedKVLayer(SWAKVCacheLayer):
    """Window cache + ``len(stream_dims)`` compressed-block streams sharing one h-buffer."""

    def __init__(self, max_seq_len: int, hidden_dim: int, head_dim: int, compression_rate: int,
                 stream_dims: tuple[int, ...], *, batch_size: int = 1, device: torch.device | str | None = None,
                 dtype: torch.dtype = torch.float32, keep_history: bool = False) -> None:
        if compression_rate <= 0:
            raise ValueError(f"compression_rate must be positive; got {compression_rate}")
        super().__init__(max_seq_len, head_dim, batch_size=batch_size, device=device, dtype=dtype)
        self.hidden_dim, self.compression_rate = hidden_dim, compression_rate
        self.keep_history = keep_history
        max_blocks = max_seq_len // compression_rate
        self.streams = [torch.zeros(batch_size, max_blocks, d, device=device, dtype=dtype) for d in stream_dims]
        self.h = torch.zeros(batch_size, max_seq_len if keep_history else compression_rate, hidden_dim,
                             device=device, dtype=dtype)
        self.n_blocks = 0

    def _h_origin(self) -> int:
        """Absolute position of ``self.h[:, 0]``."""
        return 0 if self.keep_history else self.n_blocks * self.compression_rate

    @property
    def h_buf_count(self) -> int:
        return self.length - self.n_blocks * self.compression_rate

    @property
    def h_buffer(self) -> Tensor:
        """The raw hidden states of the unfinished block."""
        s = self.n_blocks * self.compression_rate - self._h_origin()
        return self.h[:, s:s + self.h_buf_count]

    def _append_streams(self, h_new: Tensor, k_new: Tensor, v_new: Tensor,
                        compressors: tuple[Callable[[Tensor], Tensor], ...]) -> None:
        _check3(h_new, k_new, v_new)
        m, n = self.compression_rate, k_new.shape[1]
        self._write_window(k_new, v_new)
        if self.keep_history:
            self.h[:, self.length:self.length + n] = h_new
            raw = self.h[:, self.n_blocks * m:((self.length + n) // m) * m]
        else:
            raw = torch.cat([self.h[:, :self.h_buf_count], h_new], dim=1)
        self.length += n
        done = self.length // m
        if done > self.n_blocks:
            blocks_raw = raw[:, :(done - self.n_blocks) * m]
            for buf, comp in zip(self.streams, compressors, strict=True):
                blocks = comp(blocks_raw)
                if blocks.shape[1] != done - self.n_blocks:
                    raise RuntimeError(f"compressor returned {blocks.shape[1]} blocks, expected "
                                       f"{done - self.n_blocks}")
                buf[:, self.n_blocks:done] = blocks
        if not self.keep_history:
            left = self.length - done * m
            if left:
                self.h[:, :left] = raw[:, raw.shape[1] - left:]
        self.n_blocks = done

    def truncate(self, length: int) -> None:
        m = self.compression_rate
        if not self.keep_history:
            if length < self.n_blocks * m:
                raise RuntimeError("rolling back across an emitted compressed block needs keep_history=True")
            super().truncate(length)
            return
        super().truncate(length)
        self.n_blocks = min(self.n_blocks, length // m)

    def reset(self) -> None:
        super().reset()
        self.n_blocks = 0

    def _buffers(self) -> list[Tensor]:
        return [self.k, self.v, self.h, *self.streams]


class HCAKVCacheLayer(CompressedKVLayer):
    def __init__(self, max_seq_len: int, hidden_dim: int, head_dim: int, compression_rate: int, *,
                 batch_size: int = 1, device: torch.device | str | None = None,
                 dtype: torch.dtype = torch.float32, keep_history: bool = False) -> None:
        super().__init__(max_seq_len, hidden_dim, head_dim, compression_rate, (head_dim,), batch_size=batch_size,
                         device=device, dtype=dtype, keep_history=keep_history)

    @property
    def compressed(self) -> Tensor:
        return self.streams[0]

    def append(self, h_new: Tensor, sw_k_new: Tensor, sw_v_new: Tensor, *,  # type: ignore[override]
               compressor: Callable[[Tensor], Tensor]) -> tuple[Tensor, Tensor, Tensor]:
        self._append_streams(h_new, sw_k_new, sw_v_new, (compressor,))
        return self.streams[0][:, :self.n_blocks], self.k[:, :self.length], self.v[:, :self.length]


class CSAKVCacheLayer(CompressedKVLayer):
    def __init__(self, max_seq_len: int, hidden_dim: int, head_dim: int, c_indexer: int, compression_rate: int, *,
                 batch_size: int = 1, device: torch.device | str | None = None,
                 dtype: torch.dtype = torch.float32, keep_history: bool = False) -> None:
        super().__init__(max_seq_len, hidden_dim, head_dim, compression_rate, (head_dim, c_indexer),
                         batch_size=batch_size, device=device, dtype=dtype, keep_history=keep_history)
        self.c_indexer = c_indexer

    @property
    def compressed_kv(self) -> Tensor:
        return self.streams[0]

    @property
    def indexer_kv(self) -> Tensor:
        return self.streams[1]

    def append(self, h_new: Tensor, sw_k_new: Tensor, sw_v_new: Tensor, *,  # type: ignore[override]
               compressor: Callable[[Tensor], Tensor],
               indexer_compressor: Callable[[Tensor], Tensor]) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        self._append_streams(h_new, sw_k_new, sw_v_new, (compressor, indexer_compressor))
        nb, t = self.n_blocks, self.length
        return self.streams[0][:, :nb], self.streams[1][:, :nb], self.k[:, :t], self.v[:, :t]


CacheLayer = SWAKVCacheLayer | HCAKVCacheLayer | CSAKVCacheLayer | None


class KVCacheBundle:
    """Per-block cache list; ``None`` entries mean "recompute this block"."""

    def __init__(self, layers: list[CacheLayer]) -> None:
        self._layers = list(layers)

    def __len__(self) -> int:
        return len(self._layers)

    def for_layer(self, idx: int) -> CacheLayer:
        return self._layers[idx]

    @property
    def length(self) -> int:
        return next((layer.length for layer in self._layers if layer is not None), 0)

    def reset(self) -> None:
        for layer in self._layers:
            if layer is not None:
                layer.reset()

    def truncate(self, length: int) -> None:
        for layer in self._layers:
            if layer is not None:
                layer.truncate(length)

    def nbytes(self) -> int:
        return sum(layer.nbytes() for layer in self._layers if layer is not None)

    @classmethod
    def for_model(cls, model: object, *, max_seq_len: int, batch_size: int = 1,
                  device: torch.device | str | None = None, dtype: torch.dtype | None = None,
                  keep_history: bool = False) -> KVCacheBundle:
        """One cache per block by attention type; dtype/device default to the model's."""
        from saint_llm_b200.models.attention import CSA, HCA, NSAttention, SWAttention

        cfg = model.cfg  # type: ignore[attr-defined]
        p = next(model.parameters())  # type: ignore[attr-defined]
        dev = p.device if device is None else device
        dt = p.dtype if dtype is None else dtype
        hd, d = cfg.attention.head_dim, cfg.hidden_dim
        kw = {"batch_size": batch_size, "device": dev, "dtype": dt}
        ckw = {**kw, "keep_history": keep_history}
        layers: list[CacheLayer] = []
        for block in model.blocks:  # type: ignore[attr-defined]
            a = block.attention
            if isinstance(a, CSA):
                layers.append(CSAKVCacheLayer(max_seq_len, d, hd, cfg.csa.indexer_head_dim, cfg.csa.compression_rate,
                                              **ckw))
            elif isinstance(a, HCA):
                layers.append(HCAKVCacheLayer(max_seq_len, d, hd, cfg.hca.compression_rate, **ckw))
            elif isinstance(a, (SWAttention, NSAttention)):
                layers.append(SWAKVCacheLayer(max_seq_len, hd, **kw))
            else:
                layers.append(None)
        return cls(layers)


__all__ = ["CSAKVCacheLayer", "CacheLayer", "CompressedKVLayer", "HCAKVCacheLayer", "KVCacheBundle",
           "SWAKVCacheLayer"]

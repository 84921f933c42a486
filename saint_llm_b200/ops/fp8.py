"""Block-scaled FP8 on the tensor cores: quantisation kernels and the tcgen05 GEMM.

``quantize_rows(x)`` quantises activations in 1 x 128 blocks, ``quantize_blocks(w)``
weights in 128 x 128 blocks; both give E4M3 values with power-of-two scales (the
smallest 2^e with amax / 2^e <= 448).  ``gemm(a, b)`` computes
``dequant(a) @ dequant(b)^T`` in bf16 with the block scales applied inside the MMA
(``tcgen05.mma kind::mxf8f6f4.block_scale``), so the operands stay FP8 all the way.

The reference quantises the same way in eager PyTorch (``kernels/quant/reference.py:32-134``)
and runs its real FP8 forward through ``torch._scaled_mm`` with rowwise / per-channel
scales (``kernels/fp8_gemm.py:24-101``).  On CPU (and under ``backend.eager_mode``) the
functions here run the PyTorch oracle of the same recipe: identical E4M3 bytes and scales,
an fp32 product of the dequantised operands.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from saint_llm_b200.ops import backend
from saint_llm_b200.ops.gemm import error_word
from saint_llm_b200.ops.quant import E4M3_MAX, pow2_scale

BLOCK = 128


@dataclass
class Fp8Operand:
    """E4M3 values (R, K) as bytes, fp32 block scales, and (native only) the scale-factor
    bytes in the layout the GEMM copies into tensor memory."""

    q: Tensor
    scale: Tensor
    sf: Tensor | None
    kind: str  # "rows" (scale (R, K/128)) or "blocks" (scale (R/128, K/128))

    @property
    def shape(self) -> torch.Size:
        return self.q.shape

    def dequantize(self) -> Tensor:
        r, k = self.q.shape
        v = self.q.view(torch.float8_e4m3fn).float()
        if self.kind == "rows":
            return (v.reshape(r, k // BLOCK, BLOCK) * self.scale[..., None]).reshape(r, k)
        return (v.reshape(r // BLOCK, BLOCK, k // BLOCK, BLOCK) * self.scale[:, None, :, None]).reshape(r, k)


def _oracle_rows(x: Tensor) -> Fp8Operand:
    m, k = x.shape
    xb = x.float().reshape(m, k // BLOCK, BLOCK)
    s = pow2_scale(xb.abs().amax(-1))
    q = (xb / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).reshape(m, k)
    return Fp8Operand(q.view(torch.uint8), s, None, "rows")


def _oracle_blocks(w: Tensor) -> Fp8Operand:
    n, k = w.shape
    wb = w.float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    s = pow2_scale(wb.abs().amax(dim=(1, 3)))
    q = (wb / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).reshape(n, k)
    return Fp8Operand(q.view(torch.uint8), s, None, "blocks")


def _check(t: Tensor, rows_mult: int) -> None:
    if t.dim() != 2 or t.shape[-1] % BLOCK or t.shape[0] % rows_mult:
        raise ValueError(f"FP8 operand {tuple(t.shape)} must be 2-D with K % 128 == 0"
                         + (" and rows % 128 == 0" if rows_mult > 1 else ""))


def quantize_rows(x: Tensor) -> Fp8Operand:
    """1 x 128 activation quantisation of (M, K)."""
    _check(x, 1)
    if not backend.native_for(x):
        return _oracle_rows(x)
    x = x.to(torch.bfloat16)
    if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.uint8, device=x.device)
    sf = torch.empty(backend.ext().fp8_sf_bytes(m, k), dtype=torch.uint8, device=x.device)
    scale = torch.empty((m, k // BLOCK), dtype=torch.float32, device=x.device)
    backend.ext().fp8_quant_rows(x, q, sf, scale)
    return Fp8Operand(q, scale, sf, "rows")


def quantize_blocks(w: Tensor) -> Fp8Operand:
    """128 x 128 weight quantisation of (N, K)."""
    _check(w, BLOCK)
    if not backend.native_for(w):
        return _oracle_blocks(w)
    w = w.to(torch.bfloat16)
    if w.stride(-1) != 1 or w.stride(0) % 8 or w.data_ptr() % 16:
        w = w.contiguous()
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.uint8, device=w.device)
    sf = torch.empty(backend.ext().fp8_sf_bytes(n, k), dtype=torch.uint8, device=w.device)
    scale = torch.empty((n // BLOCK, k // BLOCK), dtype=torch.float32, device=w.device)
    backend.ext().fp8_quant_blocks(w, q, sf, scale)
    return Fp8Operand(q, scale, sf, "blocks")


def gemm(a: Fp8Operand, b: Fp8Operand) -> Tensor:
    """bf16 (M, N) = dequant(a) @ dequant(b)^T; ``a`` from ``quantize_rows``, ``b`` from
    ``quantize_blocks`` (N % 128 == 0)."""
    if a.shape[1] != b.shape[1]:
        raise ValueError(f"K mismatch: {tuple(a.shape)} vs {tuple(b.shape)}")
    if a.sf is None or b.sf is None or not a.q.is_cuda or not backend.native_for(a.q):
        return (a.dequantize() @ b.dequantize().t()).to(torch.bfloat16)
    out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16, device=a.q.device)
    backend.ext().gemm_fp8(a.q, a.sf, b.q, b.sf, out, error_word(a.q.device))
    return out


def linear(x: Tensor, w: Tensor) -> Tensor:
    """``x @ w^T`` with the block-scaled FP8 recipe (x: (..., K), w: (N, K))."""
    k = x.shape[-1]
    y = gemm(quantize_rows(x.reshape(-1, k)), quantize_blocks(w))
    return y.reshape(*x.shape[:-1], w.shape[0])


__all__ = ["BLOCK", "Fp8Operand", "gemm", "linear", "quantize_blocks", "quantize_rows"]


# ---------------------------------------------------------------- training weight cache
_EPOCH = [0]


def bump_weight_epoch() -> None:
    """Mark every cached FP8 weight stale (the optimizer updated the bf16 weights in place;
    native optimizer kernels do not move torch's version counters)."""
    _EPOCH[0] += 1


def weight_epoch() -> int:
    return _EPOCH[0]


class Fp8WeightCache:
    """Block-scaled FP8 copy of one weight matrix (or a fixed arrangement of several) kept in
    persistent buffers and re-quantised in place when the weights change.

    ``kind``: "rows" -- ``sources`` stacked along the output dimension (2-D (N_i, K) each, or
    one 3-D (E, N, K) pool flattened to (E * N, K)); "cols" -- 2-D (N, K_i) sources joined
    along K; "gu" -- the gate and up weights of a SwiGLU pool (two (E, I, K) tensors, or E
    gate then E up (I, K) matrices), quantised into the interleaved 64-row layout of the FP8
    SwiGLU epilogue.  Every piece spans whole 128 x 128 blocks, so quantising the arrangement
    equals quantising each piece alone.

    The buffers never move, so a CUDA graph that reads them stays valid across steps: the
    training step refreshes every cache once after the optimizer (``refresh_all``), outside
    any capture.  ``get()`` refreshes lazily when the weights changed since the last refresh
    (the epoch moved, or a weight's version counter did) and no capture is running."""

    _live: list = []

    def __init__(self, sources: list[Tensor], kind: str = "rows") -> None:
        import weakref

        self.sources = list(sources)
        self.kind = kind
        dev = sources[0].device
        if kind == "gu":
            if sources[0].dim() == 3:
                e, i, k = sources[0].shape
            else:
                e, (i, k) = len(sources) // 2, sources[0].shape
            n = e * 2 * i
        elif kind == "cols":
            n, k = sources[0].shape[0], sum(s.shape[1] for s in sources)
        else:
            k = sources[0].shape[-1]
            n = sum(s.numel() // k for s in sources)
        if n % BLOCK or k % BLOCK:
            raise ValueError(f"FP8 weight cache needs rows and K multiples of 128 (got {n} x {k})")
        self.shape = (n, k)
        self.q = torch.empty((n, k), dtype=torch.uint8, device=dev)
        self.sf = torch.empty(backend.ext().fp8_sf_bytes(n, k), dtype=torch.uint8, device=dev)
        self._stamp: tuple | None = None
        Fp8WeightCache._live.append(weakref.ref(self))

    def _current(self) -> tuple:
        return (_EPOCH[0], *(s._version for s in self.sources))

    def refresh(self) -> None:
        ext = backend.ext()
        with torch.no_grad():
            src = [s.detach().to(torch.bfloat16) for s in self.sources]
            if self.kind == "gu":
                if src[0].dim() == 3:
                    wg, wu = src[0].contiguous(), src[1].contiguous()
                else:
                    e = len(src) // 2
                    wg, wu = torch.stack(src[:e]), torch.stack(src[e:])
                ext.fp8_quant_blocks_gu(wg, wu, self.q, self.sf)
                self._stamp = self._current()
                return
            if self.kind == "cols":
                w = src[0].contiguous() if len(src) == 1 else torch.cat(src, 1)
            else:
                k = src[0].shape[-1]
                flat = [t.reshape(-1, k) for t in src]
                w = flat[0].contiguous() if len(flat) == 1 else torch.cat(flat, 0)
            ext.fp8_quant_blocks(w, self.q, self.sf, None)
        self._stamp = self._current()

    def get(self) -> Fp8Operand:
        if self._stamp != self._current() and not torch.cuda.is_current_stream_capturing():
            self.refresh()
        return Fp8Operand(self.q, torch.empty(0), self.sf, "blocks")

    @classmethod
    def refresh_all(cls) -> int:
        """Re-quantise every live cache whose weights changed; returns how many."""
        n = 0
        alive = []
        for ref in cls._live:
            c = ref()
            if c is None:
                continue
            alive.append(ref)
            if c._stamp != c._current():
                c.refresh()
                n += 1
        cls._live = alive
        return n


def transient_weight(sources: list[Tensor], kind: str = "rows") -> Fp8Operand:
    """Quantise now into fresh buffers (no cache): for weights whose FP8 copy would not fit
    next to the training state."""
    c = Fp8WeightCache(sources, kind)
    c.refresh()
    Fp8WeightCache._live.pop()  # not tracked: it dies with the caller
    return Fp8Operand(c.q, torch.empty(0), c.sf, "blocks")


def cached_weight(owner: object, attr: str, sources: list[Tensor], kind: str = "rows") -> Fp8Operand:
    """The FP8 copy of ``sources`` cached on ``owner`` (a module) under ``attr``."""
    cache = getattr(owner, attr, None)
    if cache is None or len(cache.sources) != len(sources) or any(
            a is not b for a, b in zip(cache.sources, sources, strict=True)):
        cache = Fp8WeightCache(sources, kind)
        object.__setattr__(owner, attr, cache)  # not a submodule / parameter
    return cache.get()


def gather_quantize_rows(h: Tensor, row_token: Tensor, rows: int) -> Fp8Operand:
    """1 x 128 quantisation of the gathered rows ``h[row_token[r]]`` (zero for -1), r < rows."""
    from saint_llm_b200.ops.gemm import error_word

    h = h.to(torch.bfloat16).contiguous()
    k = h.shape[1]
    q = torch.empty((rows, k), dtype=torch.uint8, device=h.device)
    sf = torch.empty(backend.ext().fp8_sf_bytes(rows, k), dtype=torch.uint8, device=h.device)
    backend.ext().fp8_gather_quant_rows(h, row_token, q, sf, error_word(h.device))
    return Fp8Operand(q, torch.empty(0), sf, "rows")


__all__ += ["Fp8WeightCache", "bump_weight_epoch", "cached_weight", "gather_quantize_rows", "transient_weight",
            "weight_epoch"]

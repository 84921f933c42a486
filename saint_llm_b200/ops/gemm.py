"""Python entry points of the native tcgen05 GEMM.

``gemm_nt(a, b)`` computes ``a @ b^T`` for logical a (..., M, K) and b (..., N, K)
with any layout whose last or second-to-last stride is 1: a unit stride along K is
passed as a K-major operand, a unit stride along M/N as an MN-major operand (the
tensor cores read both directly, no transposes are materialised).  Inputs are bf16;
outputs bf16 or fp32, optionally accumulated (``out += a @ b^T``, fp32).

K must be a multiple of 64; other K are zero-padded here (a correct, slower path
used only by tiny test shapes).  TMA needs 16-byte aligned bases and row strides;
non-conforming operands are copied to a conforming layout first.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from saint_llm_b200.ops import backend

_ERR: dict[int, Tensor] = {}


def error_word(device: torch.device) -> Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[idx] = t
    return t


ERROR_NAMES = {1: "timeout waiting for a TMA stage", 2: "timeout waiting for a free stage",
               3: "timeout waiting for a TMEM accumulator", 4: "bad shape", 5: "peer timeout",
               6: "index out of bounds", 7: "expert-parallel receive capacity exceeded"}


def check_errors(device: torch.device | None = None) -> None:
    """Raise if any native kernel recorded an error on ``device`` (host sync)."""
    devs = [device] if device is not None else [torch.device("cuda", i) for i in _ERR]
    for d in devs:
        w = error_word(d)
        code = int(w.item())
        if code:
            w.zero_()
            raise RuntimeError(f"native kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")


def _aligned(t: Tensor) -> bool:
    if t.data_ptr() % 16:
        return False
    if t.dim() >= 2 and t.shape[-2] > 1 and (t.stride(-2) * t.element_size()) % 16:
        return False
    return not (t.dim() == 3 and t.shape[0] > 1 and (t.stride(0) * t.element_size()) % 16)


def _as_operand(x: Tensor) -> tuple[Tensor, bool]:
    """Return (view with unit inner stride, is_mn_major) for a logical (.., R, K) operand."""
    if x.stride(-1) == 1 and _aligned(x):
        return x, False
    xt = x.transpose(-1, -2)
    if xt.stride(-1) == 1 and _aligned(xt):
        return xt, True
    return x.contiguous(), False


def gemm_nt(a: Tensor, b: Tensor, *, out: Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
            accumulate: bool = False, alpha: float = 1.0, symmetric: bool = False) -> Tensor:
    """``symmetric=True``: the caller guarantees ``a @ b^T`` is symmetric (e.g. ``b is a``);
    only tiles on or above the diagonal are multiplied, and their epilogue writes the
    transposed values into the skipped tiles below it."""
    if a.dtype != torch.bfloat16:
        a = a.to(torch.bfloat16)
    if b.dtype != torch.bfloat16:
        b = b.to(torch.bfloat16)
    k = a.shape[-1]
    if k % 64:
        pad = 64 - k % 64
        a = F.pad(a, (0, pad))
        b = F.pad(b, (0, pad))
    squeeze = False
    if a.dim() == 2 and b.dim() == 3:
        a = a.unsqueeze(0).expand(b.shape[0], *a.shape)
    if a.dim() == 3 and b.dim() == 2:
        b = b.unsqueeze(0).expand(a.shape[0], *b.shape)
    if a.dim() == 3 and (a.stride(0) == 0 or b.stride(0) == 0):
        a, b = a.contiguous(), b.contiguous()
    m, n = a.shape[-2], b.shape[-2]
    shape = (*a.shape[:-2], m, n)
    if out is None:
        if accumulate:
            raise ValueError("accumulate needs an output tensor")
        out = torch.empty(shape, dtype=out_dtype, device=a.device)
    elif out.stride(-1) != 1:
        raise ValueError("output needs a unit inner stride")
    if m == 0 or n == 0:
        return out
    av, a_mn = _as_operand(a)
    bv, b_mn = _as_operand(b)
    if av.dim() == 2 and a.dim() == 2:
        squeeze = False
    sym = symmetric and not accumulate
    # symmetric: the GEMM computes the tiles on and above the diagonal and writes their
    # transposes into the skipped ones from its epilogue (no mirror pass)
    backend.ext().gemm(av, bv, out, a_mn, b_mn, accumulate, float(alpha), error_word(a.device), sym)
    del squeeze
    return out


def gemm_axpby(a: Tensor, b: Tensor, c: Tensor, *, alpha: float = 1.0, beta: float = 1.0,
               symmetric: bool = False) -> Tensor:
    """``alpha * a @ b^T + beta * c`` in one GEMM pass (bf16 in/out, fp32 accumulation);
    ``symmetric=True`` when the result is symmetric (see ``gemm_nt``)."""
    a, b = a.to(torch.bfloat16), b.to(torch.bfloat16)
    k = a.shape[-1]
    if k % 64:
        pad = 64 - k % 64
        a, b = F.pad(a, (0, pad)), F.pad(b, (0, pad))
    c = c.to(torch.bfloat16).contiguous()
    out = torch.empty_like(c)
    av, a_mn = _as_operand(a)
    bv, b_mn = _as_operand(b)
    backend.ext().gemm_axpby(av, bv, c, out, a_mn, b_mn, float(alpha), float(beta), error_word(a.device), symmetric)
    return out


def matmul(a: Tensor, b: Tensor, *, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """``a @ b`` for (.., M, K) x (.., K, N)."""
    return gemm_nt(a, b.transpose(-1, -2), out_dtype=out_dtype)


def bmm(a: Tensor, b: Tensor) -> Tensor:
    """Batched ``a @ b`` with fp32 output (Newton-Schulz helper)."""
    return gemm_nt(a, b.transpose(-1, -2), out_dtype=torch.float32)


def grouped_mm(a: Tensor, b: Tensor, offsets: Tensor) -> Tensor:
    """a (M, K) rows grouped by cumulative ``offsets``; b (E, K, N) -> (M, N).

    Generic ragged path (used by ``GroupedSwiGLUExperts`` outside the fused MoE
    layer): one native GEMM per non-empty group.
    """
    out = torch.empty(a.shape[0], b.shape[2], dtype=torch.bfloat16, device=a.device)
    start = 0
    for e, end in enumerate(offsets.tolist()):
        if end > start:
            gemm_nt(a[start:end], b[e].transpose(0, 1), out=out[start:end])
        start = end
    return out.to(a.dtype)


__all__ = ["bmm", "check_errors", "error_word", "gemm_axpby", "gemm_nt", "grouped_mm", "matmul"]

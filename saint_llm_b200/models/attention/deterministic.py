"""Batch-invariant attention and a deterministic-mode context (reference
``core/attention/deterministic.py:39-153``).

``batch_invariant_attention`` is unfused fp32 ``softmax(QK^T * scale + mask) V``: every
output row depends only on its own inputs (no tiling whose boundaries move with the batch
or padding).  Fully masked rows output zero.  ``is_causal`` uses the bottom-right
alignment of ``F.scaled_dot_product_attention`` (query ``i`` sees key ``j`` iff
``j <= i + Lk - Lq``).

``deterministic_mode`` turns on deterministic algorithms, disables cuDNN autotuning and
sets ``CUBLAS_WORKSPACE_CONFIG`` (needed by cuBLAS to stay on one algorithm) for the body,
restoring every previous value on exit, even when the body raises.
"""

from __future__ import annotations

import contextlib
import math
import os
from collections.abc import Iterator

import torch
from torch import Tensor

_CUBLAS_ENV = "CUBLAS_WORKSPACE_CONFIG"


@contextlib.contextmanager
def deterministic_mode(*, warn_only: bool = False) -> Iterator[None]:
    saved = (torch.are_deterministic_algorithms_enabled(), torch.is_deterministic_algorithms_warn_only_enabled(),
             torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark, os.environ.get(_CUBLAS_ENV))
    if saved[4] is None:
        os.environ[_CUBLAS_ENV] = ":4096:8"
    torch.use_deterministic_algorithms(True, warn_only=warn_only)
    torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = True, False
    try:
        yield
    finally:
        torch.use_deterministic_algorithms(saved[0], warn_only=saved[1])
        torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = saved[2], saved[3]
        if saved[4] is None:
            os.environ.pop(_CUBLAS_ENV, None)
        else:
            os.environ[_CUBLAS_ENV] = saved[4]


def batch_invariant_attention(q: Tensor, k: Tensor, v: Tensor, *, attn_mask: Tensor | None = None,
                              scale: float | None = None, is_causal: bool = False) -> Tensor:
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    lq, lk = s.shape[-2], s.shape[-1]
    visible = torch.ones(lq, lk, dtype=torch.bool, device=s.device)
    if is_causal:
        visible = torch.ones_like(visible).tril(lk - lq)
    if attn_mask is not None and attn_mask.dtype == torch.bool:
        visible = visible & attn_mask
    elif attn_mask is not None:
        s = s + attn_mask.float()
    s = s.masked_fill(~visible, float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return torch.matmul(p, v.float()).to(q.dtype)


__all__ = ["batch_invariant_attention", "deterministic_mode"]

"""Token embedding whose backward adds the used rows straight into ``weight.main_grad``.

Autograd's embedding backward materialises a dense ``(vocab, dim)`` gradient every
micro-batch (134 MB for a 32k x 2k table) that the mixed-precision engine then adds into
the fp32 ``main_grad`` (another ~0.8 GB of traffic).  Only ``tokens`` rows are non-zero,
so this backward scatters ``tokens x dim`` values into ``main_grad`` and returns no
weight gradient.  Without a ``main_grad`` buffer it falls back to autograd's embedding.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor


class _EmbeddingToMainGrad(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids: Tensor, weight: Tensor) -> Tensor:  # type: ignore[override]
        ctx.save_for_backward(ids)
        ctx.weight = weight
        return F.embedding(ids, weight)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        (ids,) = ctx.saved_tensors
        mg = ctx.weight.main_grad
        mg.index_add_(0, ids.reshape(-1), g.reshape(-1, g.shape[-1]).to(mg.dtype))
        return None, None


def embedding(ids: Tensor, weight: Tensor) -> Tensor:
    if getattr(weight, "main_grad", None) is not None and weight.requires_grad and torch.is_grad_enabled():
        return _EmbeddingToMainGrad.apply(ids, weight)
    return F.embedding(ids, weight)


__all__ = ["embedding"]

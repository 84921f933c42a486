"""Hybrid Newton-Schulz orthogonalisation for Muon.

Reference semantics (``optim/newton_schulz.py:20-57``): fp32, Frobenius-normalise
with eps 1e-7, run on the tall orientation, 8 iterations with (3.4445, -4.7750,
2.0315) then 2 with (2, -1.5, 0.5), each ``X <- aX + b(XX^T)X + c(XX^T)^2 X``.

Because ``p(XX^T) X == X p(X^T X)``, the iteration can use either Gram matrix.  The
reference forms the Gram of the *larger* dimension; ``hybrid_newton_schulz`` keeps
that orientation (bit-for-bit oracle), while ``batched_newton_schulz`` -- the one the
optimizer runs -- uses the smaller Gram ``X^T X`` (for a tall X) and stacks every
matrix of one shape into a single batch.  On CUDA it runs on the native batched
tensor-core GEMM with bf16 operands and fp32 accumulation (``precision="bf16"``);
``precision="fp32"`` keeps everything in fp32 for parity tests.
"""

from __future__ import annotations

import torch
from torch import Tensor

STAGE1 = (3.4445, -4.7750, 2.0315)
STAGE2 = (2.0, -1.5, 0.5)


def hybrid_newton_schulz(matrix: Tensor, n_iter_stage1: int = 8, n_iter_stage2: int = 2,
                         coeffs_stage1: tuple[float, float, float] = STAGE1,
                         coeffs_stage2: tuple[float, float, float] = STAGE2,
                         eps: float = 1.0e-7) -> Tensor:
    dtype = matrix.dtype
    x = matrix.float()
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + eps)
    flip = x.shape[-2] < x.shape[-1]
    if flip:
        x = x.transpose(-2, -1)
    for n, (a, b, c) in ((n_iter_stage1, coeffs_stage1), (n_iter_stage2, coeffs_stage2)):
        for _ in range(n):
            g = x @ x.transpose(-2, -1)
            x = a * x + b * (g @ x) + c * (g @ g @ x)
    if flip:
        x = x.transpose(-2, -1)
    return x.to(dtype)


def _bmm(a: Tensor, b: Tensor, precision: str) -> Tensor:
    if a.is_cuda and precision == "bf16":
        from saint_llm_b200.ops import backend

        if backend.native_for(a):
            from saint_llm_b200.ops import gemm

            return gemm.bmm(a, b)
    return torch.matmul(a, b)


def batched_newton_schulz(x: Tensor, n_iter_stage1: int = 8, n_iter_stage2: int = 2,
                          coeffs_stage1: tuple[float, float, float] = STAGE1,
                          coeffs_stage2: tuple[float, float, float] = STAGE2,
                          eps: float = 1.0e-7, precision: str = "bf16") -> Tensor:
    """Orthogonalise a batch (..., n, m) using the small Gram matrix.

    Output dtype = input dtype.  ``precision="bf16"`` keeps X in bf16 between
    iterations (fp32 accumulation inside each GEMM); ``"fp32"`` keeps fp32.
    """
    dtype = x.dtype
    lead = x.shape[:-2]
    n, m = x.shape[-2:]
    y = x.reshape(-1, n, m).float()
    y = y / (torch.linalg.vector_norm(y, dim=(-2, -1), keepdim=True) + eps)
    wide = n < m
    if not wide:  # make it wide: rows <= cols, Gram = Y Y^T is the small one
        y = y.transpose(-2, -1)
    work = torch.bfloat16 if precision == "bf16" and y.is_cuda else torch.float32
    y = y.to(work).contiguous()
    for steps, (a, b, c) in ((n_iter_stage1, coeffs_stage1), (n_iter_stage2, coeffs_stage2)):
        for _ in range(steps):
            g = _bmm(y, y.transpose(-2, -1), precision)          # (B, r, r) fp32-accumulated
            p = b * g + c * _bmm(g.to(work), g.to(work), precision)  # b G + c G^2
            y = (a * y.float() + _bmm(p.to(work), y, precision).float()).to(work)
    if not wide:
        y = y.transpose(-2, -1)
    return y.reshape(*lead, n, m).to(dtype)


def native_newton_schulz(y: Tensor, n_iter_stage1: int = 8, n_iter_stage2: int = 2,
                         coeffs_stage1: tuple[float, float, float] = STAGE1,
                         coeffs_stage2: tuple[float, float, float] = STAGE2) -> Tensor:
    """Newton-Schulz on already-normalised bf16 matrices (B, r, c), three fused GEMMs per step.

    Wide (r <= c):  G = Y Y^T ;  P = c G G + b G ;  Y <- P Y + a Y
    Tall (r > c):   G = Y^T Y ;  P = c G G + b G ;  Y <- Y P + a Y
    The "+ b G" and "+ a Y" terms ride in the GEMM epilogue (no element-wise passes),
    and neither orientation needs a transpose copy: the tensor cores read Y^T directly.
    G and P are symmetric: their GEMMs skip the tiles below the diagonal (~40 % of the
    tiles of a 1408 x 1408 Gram) and fill them from the epilogue of the tiles they mirror.
    """
    from saint_llm_b200.ops import gemm

    wide = y.shape[-2] <= y.shape[-1]
    for steps, (a, b, c) in ((n_iter_stage1, coeffs_stage1), (n_iter_stage2, coeffs_stage2)):
        for _ in range(steps):
            if wide:
                g = gemm.gemm_nt(y, y, symmetric=True)
                p = gemm.gemm_axpby(g, g, g, alpha=c, beta=b, symmetric=True)
                y = gemm.gemm_axpby(p, y.transpose(-1, -2), y, alpha=1.0, beta=a)
            else:
                yt = y.transpose(-1, -2)
                g = gemm.gemm_nt(yt, yt, symmetric=True)
                p = gemm.gemm_axpby(g, g, g, alpha=c, beta=b, symmetric=True)
                y = gemm.gemm_axpby(y, p, y, alpha=1.0, beta=a)
    return y


__all__ = ["STAGE1", "STAGE2", "batched_newton_schulz", "hybrid_newton_schulz", "native_newton_schulz"]

"""Manifold-constrained hyper-connections (mHC).

The residual stream is X in (B, T, n, D).  Per wrapped sub-layer (reference
``core/residual/mhc.py:54-144``):

    Xn   = RMSNorm(flatten(X))                         (over n*D, eps = rms_norm_eps)
    A    = sigmoid(alpha_pre  * Xn W_pre^T  + s_pre)     (n,)
    B    = Sinkhorn(alpha_res * Xn W_res^T  + s_res)     (n, n), ``iters`` alternating
                                                        row/column normalisations of
                                                        exp(x - max) with +1e-12
    C    = 2 sigmoid(alpha_post * Xn W_post^T + s_post)  (n,)
    in   = sum_h A_h X_h ;   X' = B X + C (x) F(in)

``W_*`` start at zero.  On CUDA ``split``/``combine`` run as fused sm_100a kernels
(``ops.mhc``): one pass over X computes the norm statistics, the 2n+n^2 gate
projections, the Sinkhorn iterations in registers and the A-weighted mix; the
combine is one pass as well.  The eager code below is the oracle.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from saint_llm_b200.config import MHCConfig
from saint_llm_b200.models.attention.common import RMSNorm
from saint_llm_b200.ops import backend


def sinkhorn_knopp(logits: Tensor, n_iter: int) -> Tensor:
    x = torch.exp(logits - logits.amax(dim=(-2, -1), keepdim=True))
    for _ in range(n_iter):
        x = x / (x.sum(dim=-1, keepdim=True) + 1.0e-12)
        x = x / (x.sum(dim=-2, keepdim=True) + 1.0e-12)
    return x


class MHC(nn.Module):
    def __init__(self, hidden_dim: int, cfg: MHCConfig, rms_norm_eps: float = 1.0e-6) -> None:
        super().__init__()
        n = cfg.expansion_factor
        self.hidden_dim = hidden_dim
        self.n_hc = n
        self.sinkhorn_iters = cfg.sinkhorn_iters
        flat = n * hidden_dim
        self.norm = RMSNorm(flat, eps=rms_norm_eps)
        self.w_pre = nn.Linear(flat, n, bias=False)
        self.w_res = nn.Linear(flat, n * n, bias=False)
        self.w_post = nn.Linear(flat, n, bias=False)
        self.alpha_pre = nn.Parameter(torch.full((1,), cfg.init_alpha))
        self.alpha_res = nn.Parameter(torch.full((1,), cfg.init_alpha))
        self.alpha_post = nn.Parameter(torch.full((1,), cfg.init_alpha))
        self.s_pre = nn.Parameter(torch.full((n,), cfg.init_static_bias))
        self.s_res = nn.Parameter(torch.full((n, n), cfg.init_static_bias))
        self.s_post = nn.Parameter(torch.full((n,), cfg.init_static_bias))
        for w in (self.w_pre, self.w_res, self.w_post):
            nn.init.zeros_(w.weight)

    @staticmethod
    def expand(x: Tensor, n_hc: int) -> Tensor:
        return x.unsqueeze(-2).expand(*x.shape[:-1], n_hc, x.shape[-1]).contiguous()

    @staticmethod
    def collapse(x: Tensor) -> Tensor:
        return x.mean(dim=-2)

    def _gates(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        b, t, n, d = x.shape
        xn = self.norm(x.reshape(b, t, n * d))
        a = torch.sigmoid(self.alpha_pre * self.w_pre(xn) + self.s_pre)
        bm = sinkhorn_knopp(self.alpha_res * self.w_res(xn).reshape(b, t, n, n) + self.s_res,
                            self.sinkhorn_iters)
        c = 2.0 * torch.sigmoid(self.alpha_post * self.w_post(xn) + self.s_post)
        return a, bm, c

    def split(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        if backend.native_for(x):
            from saint_llm_b200.ops import mhc as mhc_ops

            return mhc_ops.mhc_split(self, x)
        a, bm, c = self._gates(x)
        return torch.einsum("bth,bthd->btd", a, x), a, bm, c

    def combine(self, x: Tensor, inner_out: Tensor, b_l: Tensor, c_l: Tensor) -> Tensor:
        if backend.native_for(x):
            from saint_llm_b200.ops import mhc as mhc_ops

            return mhc_ops.mhc_combine(x, inner_out, b_l, c_l)
        return torch.einsum("bthk,btkd->bthd", b_l, x) + torch.einsum("bth,btd->bthd", c_l, inner_out)

    def forward(self, x: Tensor, inner: nn.Module) -> Tensor:
        inner_in, _, b_l, c_l = self.split(x)
        return self.combine(x, inner(inner_in), b_l, c_l)


__all__ = ["MHC", "sinkhorn_knopp"]

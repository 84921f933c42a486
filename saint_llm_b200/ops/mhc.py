"""mHC split / combine on the native kernels.

split (one autograd node):
    q = X W_fold^T (tcgen05 GEMM), ssq = row sums of X^2; W_fold = [w_pre; w_res; w_post] * norm.weight
    a,b,c = mhc_gates_fwd(p, alpha, s)    sigmoid / Sinkhorn (in registers) / 2 sigmoid
    inner = mhc_premix(X, a)
combine:  X' = B X + C (x) out  (mhc_combine), backward in one pass (mhc_combine_bwd).

The folding of the norm weight into the projection and the alpha / static-bias
gradients are tiny tensors handled by autograd around the node.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from saint_llm_b200.ops import backend, gemm


def _bf16c(t: Tensor) -> Tensor:
    return (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)).contiguous()


_GROUPS: dict[tuple[int, torch.device], Tensor] = {}


def _column_groups(n: int, dev: torch.device) -> Tensor:
    """Group id (0 pre, 1 res, 2 post) of each gate column, cached per device so the
    backward makes no host-to-device copy (CUDA-graph capturable)."""
    key = (n, dev)
    g = _GROUPS.get(key)
    if g is None:
        g = torch.cat([torch.full((n,), 0, dtype=torch.long), torch.full((n * n,), 1, dtype=torch.long),
                       torch.full((n,), 2, dtype=torch.long)]).to(dev)
        _GROUPS[key] = g
    return g


class _SplitFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X: Tensor, w_fold: Tensor, alpha: Tensor, s_pre: Tensor, s_res: Tensor,  # type: ignore[override]
                s_post: Tensor, n: int, iters: int, eps: float):
        b_, t_, _, d = X.shape
        T = b_ * t_
        Xf = _bf16c(X).view(T, n * d)
        P = w_fold.shape[0]
        ext = backend.ext()
        dev = X.device
        p = torch.empty(T, P, dtype=torch.float32, device=dev)
        ssq = torch.empty(T, dtype=torch.float32, device=dev)
        r = torch.empty(T, dtype=torch.float32, device=dev)
        wf = w_fold.float().contiguous()
        gemm.gemm_nt(Xf, wf.to(torch.bfloat16), out=p)  # skinny (T, P) projection, split-K on the GEMM
        ext.row_sumsq(Xf, ssq)
        al = alpha.float().contiguous()
        sp, sr, so = s_pre.float().contiguous(), s_res.float().contiguous(), s_post.float().contiguous()
        a = torch.empty(T, n, dtype=torch.float32, device=dev)
        bm = torch.empty(T, n, n, dtype=torch.float32, device=dev)
        c = torch.empty(T, n, dtype=torch.float32, device=dev)
        ext.mhc_gates_fwd(p, ssq, r, n * d, float(eps), al, sp, sr, so, a, bm, c, n, iters)
        inner = torch.empty(T, d, dtype=torch.bfloat16, device=dev)
        ext.mhc_premix(Xf, a, inner, n)
        ctx.save_for_backward(Xf, wf, al, sp, sr, so, p, r, a)
        ctx.meta = (n, iters, b_, t_, d)
        return inner.view(b_, t_, d), a.view(b_, t_, n), bm.view(b_, t_, n, n), c.view(b_, t_, n)

    @staticmethod
    def backward(ctx, d_inner: Tensor, da_out: Tensor | None, db: Tensor | None, dc: Tensor | None):  # type: ignore[override]
        Xf, wf, al, sp, sr, so, p, r, a = ctx.saved_tensors
        n, iters, b_, t_, d = ctx.meta
        T = b_ * t_
        ext = backend.ext()
        dev = Xf.device
        din = (_bf16c(d_inner).view(T, d) if d_inner is not None
               else torch.zeros(T, d, dtype=torch.bfloat16, device=dev))
        da = torch.empty(T, n, dtype=torch.float32, device=dev)
        ext.mhc_premix_da(Xf, din, da, n)
        if da_out is not None:
            da += da_out.reshape(T, n).float()
        dbf = db.reshape(T, n, n).float().contiguous() if db is not None else torch.zeros(T, n, n, device=dev)
        dcf = dc.reshape(T, n).float().contiguous() if dc is not None else torch.zeros(T, n, device=dev)
        P = p.shape[1]
        dz = torch.empty(T, P, dtype=torch.float32, device=dev)
        ext.mhc_gates_bwd(p, al, sp, sr, so, da.contiguous(), dbf, dcf, dz, n, iters)
        # z = alpha_g * p + s ; column groups: [0, n) pre, [n, n+n^2) res, [n+n^2, P) post
        grp = _column_groups(n, dev)
        dp = dz * al[grp]
        d_alpha = torch.zeros(3, dtype=torch.float32, device=dev).index_add_(0, grp, (dz * p).sum(0))
        dzs = dz.sum(0)
        d_s_pre, d_s_res, d_s_post = dzs[:n], dzs[n:n + n * n].view(n, n), dzs[n + n * n:]
        dXf = torch.empty_like(Xf)
        ext.mhc_split_bwd(dXf, Xf, din, a, dp.contiguous(), p, r, wf, n)
        dq = (dp * r[:, None]).to(torch.bfloat16)
        dW = gemm.gemm_nt(dq.t(), Xf.t(), out_dtype=torch.float32)
        return dXf.view(b_, t_, n, d), dW, d_alpha, d_s_pre, d_s_res, d_s_post, None, None, None


def mhc_split(m: nn.Module, x: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    w_fold = torch.cat([m.w_pre.weight, m.w_res.weight, m.w_post.weight], 0).float() * m.norm.weight.float()
    alpha = torch.cat([m.alpha_pre, m.alpha_res, m.alpha_post]).float()
    return _SplitFn.apply(x, w_fold, alpha, m.s_pre, m.s_res, m.s_post, m.n_hc, m.sinkhorn_iters, m.norm.eps)


class _CombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X: Tensor, out: Tensor, bm: Tensor, c: Tensor) -> Tensor:  # type: ignore[override]
        b_, t_, n, d = X.shape
        T = b_ * t_
        Xf = _bf16c(X).view(T, n * d)
        of = _bf16c(out).view(T, d)
        bf = bm.float().contiguous().view(T, n, n)
        cf = c.float().contiguous().view(T, n)
        Y = torch.empty(T, n * d, dtype=torch.bfloat16, device=X.device)
        backend.ext().mhc_combine(Xf, of, bf, cf, Y, n)
        ctx.save_for_backward(Xf, of, bf, cf)
        ctx.meta = (b_, t_, n, d)
        return Y.view(b_, t_, n, d)

    @staticmethod
    def backward(ctx, dY: Tensor):  # type: ignore[override]
        Xf, of, bf, cf = ctx.saved_tensors
        b_, t_, n, d = ctx.meta
        T = b_ * t_
        dX = torch.empty_like(Xf)
        dO = torch.empty_like(of)
        dB = torch.empty(T, n, n, dtype=torch.float32, device=Xf.device)
        dC = torch.empty(T, n, dtype=torch.float32, device=Xf.device)
        backend.ext().mhc_combine_bwd(_bf16c(dY).view(T, n * d), Xf, of, bf, cf, dX, dO, dB, dC, n)
        return dX.view(b_, t_, n, d), dO.view(b_, t_, d), dB.view(b_, t_, n, n), dC.view(b_, t_, n)


def mhc_combine(x: Tensor, inner_out: Tensor, b_l: Tensor, c_l: Tensor) -> Tensor:
    return _CombineFn.apply(x, inner_out, b_l, c_l)


__all__ = ["mhc_combine", "mhc_split"]

"""Fused LM-head + (softcap) + cross-entropy without materialising (B, T, V) logits.

Token rows are processed in chunks: logits_chunk = h_chunk W^T on the native GEMM (fp32
output), then one native kernel per row computes the (softcapped) log-sum-exp and the
target logit.  Backward recomputes each chunk's logits; a native kernel forms
``dz = scale * (softmax - onehot) * softcap'`` directly in bf16 before two native GEMMs:
``dh = dz W`` and ``dW += dz^T h`` (into ``W.main_grad`` when present).  Value and
gradients equal ``F.cross_entropy`` on the full logits (mean over rows).  ``token_logprobs`` serves GRPO-style log-probabilities.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from saint_llm_b200.ops import backend, gemm

CHUNK_ROWS = 4096


def _bf16(t: Tensor) -> Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


class _LMHeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor, weight: Tensor, target: Tensor, softcap: float | None) -> Tensor:  # type: ignore[override]
        d = h.shape[-1]
        h2 = _bf16(h.reshape(-1, d)).contiguous()
        t2 = target.reshape(-1).contiguous()
        n = h2.shape[0]
        # pad rows to a multiple of 64 once so the weight-gradient GEMM (K = rows) needs no copy
        n_pad = (n + 63) // 64 * 64
        if n_pad != n:
            h2 = F.pad(h2, (0, 0, 0, n_pad - n))
        wb = _bf16(weight)
        ext = backend.ext()
        cap = float(softcap or 0.0)
        lse_all = torch.empty(n, dtype=torch.float32, device=h.device)
        nll = torch.empty(n, dtype=torch.float32, device=h.device)
        for r0 in range(0, n, CHUNK_ROWS):
            r1 = min(n, r0 + CHUNK_ROWS)
            z = gemm.gemm_nt(h2[r0:r1], wb, out_dtype=torch.float32)
            ext.ce_fwd(z, t2[r0:r1], cap, lse_all[r0:r1], nll[r0:r1])
        ctx.save_for_backward(h2, weight, t2, lse_all)
        ctx.softcap = cap
        ctx.hshape = h.shape
        ctx.n = n
        return nll.sum() / max(n, 1)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        h2, weight, t2, lse_all = ctx.saved_tensors
        cap, n = ctx.softcap, ctx.n
        wb = _bf16(weight)
        ext = backend.ext()
        scale = (g.float() / max(n, 1)).reshape(1).contiguous()
        dh = torch.empty(n, h2.shape[1], dtype=torch.bfloat16, device=h2.device)
        mg = getattr(weight, "main_grad", None)
        dw = mg if mg is not None else torch.zeros(weight.shape, dtype=torch.float32, device=h2.device)
        for r0 in range(0, n, CHUNK_ROWS):
            r1 = min(n, r0 + CHUNK_ROWS)
            rp = min(h2.shape[0], (r1 + 63) // 64 * 64) if r1 == n else r1
            raw = gemm.gemm_nt(h2[r0:r1], wb, out_dtype=torch.float32)
            pb = torch.empty(rp - r0, raw.shape[1], dtype=torch.bfloat16, device=h2.device)
            ext.ce_bwd(raw, t2[r0:r1], lse_all[r0:r1], cap, scale, pb)  # rows past r1 are zero
            gemm.gemm_nt(pb[: r1 - r0], wb.t(), out=dh[r0:r1])
            gemm.gemm_nt(pb.t(), h2[r0:rp].t(), out=dw, accumulate=True)
        dweight = None if mg is not None else dw.to(weight.dtype)
        return dh.view(ctx.hshape), dweight, None, None


def lm_head_cross_entropy(h: Tensor, weight: Tensor, target: Tensor, *, softcap: float | None = None) -> Tensor:
    """mean over rows of CE(softcap(h W^T), target); h (.., D), weight (V, D), target (..)."""
    return _LMHeadCEFn.apply(h, weight, target, softcap)


class _TokenLogprobFn(torch.autograd.Function):
    """log p(target_r | h_r) per row, differentiable, without materialising the logits."""

    @staticmethod
    def forward(ctx, h: Tensor, weight: Tensor, target: Tensor, softcap: float | None) -> Tensor:  # type: ignore[override]
        d = h.shape[-1]
        h2 = _bf16(h.reshape(-1, d)).contiguous()
        t2 = target.reshape(-1).contiguous()
        n = h2.shape[0]
        n_pad = (n + 63) // 64 * 64
        if n_pad != n:
            h2 = F.pad(h2, (0, 0, 0, n_pad - n))
        wb = _bf16(weight)
        cap = float(softcap or 0.0)
        lse = torch.empty(n, dtype=torch.float32, device=h.device)
        nll = torch.empty(n, dtype=torch.float32, device=h.device)
        for r0 in range(0, n, CHUNK_ROWS):
            r1 = min(n, r0 + CHUNK_ROWS)
            z = gemm.gemm_nt(h2[r0:r1], wb, out_dtype=torch.float32)
            backend.ext().ce_fwd(z, t2[r0:r1], cap, lse[r0:r1], nll[r0:r1])
        ctx.save_for_backward(h2, weight, t2, lse)
        ctx.softcap, ctx.hshape, ctx.n = cap, h.shape, n
        return (-nll).view(target.shape)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        h2, weight, t2, lse = ctx.saved_tensors
        cap, n = ctx.softcap, ctx.n
        wb = _bf16(weight)
        ext = backend.ext()
        neg_g = (-g.reshape(-1).float()).contiguous()  # d logp / dz = onehot - softmax
        dh = torch.empty(n, h2.shape[1], dtype=torch.bfloat16, device=h2.device)
        mg = getattr(weight, "main_grad", None)
        dw = mg if mg is not None else torch.zeros(weight.shape, dtype=torch.float32, device=h2.device)
        for r0 in range(0, n, CHUNK_ROWS):
            r1 = min(n, r0 + CHUNK_ROWS)
            rp = min(h2.shape[0], (r1 + 63) // 64 * 64) if r1 == n else r1
            raw = gemm.gemm_nt(h2[r0:r1], wb, out_dtype=torch.float32)
            pb = torch.empty(rp - r0, raw.shape[1], dtype=torch.bfloat16, device=h2.device)
            ext.ce_bwd(raw, t2[r0:r1], lse[r0:r1], cap, neg_g[r0:r1], pb)
            gemm.gemm_nt(pb[: r1 - r0], wb.t(), out=dh[r0:r1])
            gemm.gemm_nt(pb.t(), h2[r0:rp].t(), out=dw, accumulate=True)
        dweight = None if mg is not None else dw.to(weight.dtype)
        return dh.view(ctx.hshape), dweight, None, None


def token_logprobs(h: Tensor, weight: Tensor, target: Tensor, *, softcap: float | None = None) -> Tensor:
    """log p(target) per row of ``h`` (.., D) under the LM head ``weight`` (V, D), differentiable
    with respect to ``h`` and ``weight``; the (rows, V) logits are never materialised."""
    return _TokenLogprobFn.apply(h, weight, target, softcap)


__all__ = ["lm_head_cross_entropy", "token_logprobs"]

"""CUDA training path of SWA / CSA / HCA attention.

Projections run on the native GEMM with the sibling projections of the same input
fused into one GEMM (``[q_compressor; k_proj; v_proj; w_b_kv; w_b_z]`` for attention,
``[w_dq; w_w; w_b_kv; w_b_z]`` for the indexer); Q/K RoPE+RMSNorm run as one fused
kernel per tensor in the reference's order (Q: rope then norm; K: CSA norm then rope,
SWA/HCA rope then norm).

The lightning indexer (no gradient flows through its integer output) streams token
chunks: scores = relu(q_h . k_s) weighted over heads, strict block-causal mask, top-k.

Attention itself uses a memory-bounded formulation: the sliding window is computed per
block of queries against its own and the previous key block (never a T x T score
tensor), and the CSA sparse branch is evaluated as a masked softmax over the (short)
compressed table -- exact, because the top-k picks are a subset of that table.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.ops import gemm
from saint_llm_b200.ops import linear as lin
from saint_llm_b200.ops.norm import rms_norm, rope_norm


def _bf16(t: Tensor) -> Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


class _FusedLinearFn(torch.autograd.Function):
    """y = x [W_0; W_1; ...]^T with per-weight gradients (into main_grad when present)."""

    @staticmethod
    def forward(ctx, x: Tensor, *weights: Tensor) -> Tensor:  # type: ignore[override]
        k = x.shape[-1]
        x2 = _bf16(x.reshape(-1, k))
        w = torch.cat([_bf16(wi) for wi in weights], 0)
        y = gemm.gemm_nt(x2, w)
        ctx.save_for_backward(x2, w, *weights)
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, w, *weights = ctx.saved_tensors
        dy2 = _bf16(dy.reshape(-1, w.shape[0])).contiguous()
        dx = gemm.gemm_nt(dy2, w.t()).view(*ctx.xshape)
        grads: list[Tensor | None] = [None] * len(weights)
        if any(ctx.needs_input_grad[1:]):
            dw = gemm.gemm_nt(dy2.t(), x2.t(), out_dtype=torch.float32)
            off = 0
            for i, wi in enumerate(weights):
                part = dw[off:off + wi.shape[0]]
                off += wi.shape[0]
                mg = getattr(wi, "main_grad", None)
                if mg is not None:
                    mg.add_(part)
                else:
                    grads[i] = part.to(wi.dtype)
        return (dx, *grads)


def fused_linear(x: Tensor, weights: list[Tensor]) -> Tensor:
    return _FusedLinearFn.apply(x, *weights)


def _pool(c_b: Tensor, z_b: Tensor, bias_b: Tensor, m: int) -> Tensor:
    """Softmax-over-m pooling (B, T, c) -> (B, T//m, c), fp32 math."""
    b, t, c = c_b.shape
    n = t // m
    if n == 0:
        return c_b.new_zeros(b, 0, c, dtype=torch.float32)
    z = z_b[:, : n * m].float().reshape(b, n, m, c) + bias_b.float()
    return (torch.softmax(z, dim=-2) * c_b[:, : n * m].float().reshape(b, n, m, c)).sum(-2)


def _sw_attention(q: Tensor, k: Tensor, v: Tensor, window: int, sink: Tensor | None,
                  softcap: float | None, layer: nn.Module) -> Tensor:
    """q (B,H,T,d), k/v (B,T,d): causal sliding window with per-head sink, blocked by `window`."""
    b, h, t, d = q.shape
    bq = max(16, window)
    nb = (t + bq - 1) // bq
    tp = nb * bq
    qp = F.pad(q, (0, 0, 0, tp - t)).view(b, h, nb, bq, d)
    kp = F.pad(k, (0, 0, bq, tp - t))  # one leading block of zeros
    vp = F.pad(v, (0, 0, bq, tp - t))
    kb = kp.unfold(1, 2 * bq, bq).transpose(-1, -2)  # (B, nb, 2bq, d)
    vb = vp.unfold(1, 2 * bq, bq).transpose(-1, -2)
    s = torch.matmul(qp, kb.unsqueeze(1).transpose(-1, -2)) / math.sqrt(d)  # (B,H,nb,bq,2bq)
    qpos = torch.arange(tp, device=q.device).view(nb, bq, 1)
    kpos = ((torch.arange(nb, device=q.device).view(nb, 1, 1) - 1) * bq
            + torch.arange(2 * bq, device=q.device).view(1, 1, 2 * bq))
    vis = (kpos <= qpos) & (qpos - kpos < window) & (kpos >= 0)
    with torch.no_grad():
        layer.max_attn_logit.copy_(s.detach().masked_fill(~vis, 0).abs().amax().float())
    if softcap is not None:
        s = softcap * torch.tanh(s / softcap)
    s = s.float().masked_fill(~vis, float("-inf"))
    if sink is not None:
        sk = sink.float().view(1, h, 1, 1, 1).expand(b, h, nb, bq, 1)
        p = torch.softmax(torch.cat([s, sk], -1), -1)[..., :-1]
    else:
        p = torch.softmax(s, -1)
    out = torch.matmul(p.to(vb.dtype), vb.unsqueeze(1))  # (B,H,nb,bq,d)
    return out.reshape(b, h, tp, d)[:, :, :t]


def _masked_compressed_attention(q: Tensor, kv: Tensor, mask: Tensor, sink: Tensor | None) -> Tensor:
    """q (B,H,T,d), kv (B,n,d) (K = V), mask (B|1, T, n).  Rows with nothing visible give 0."""
    d = q.shape[-1]
    s = torch.matmul(q, kv.unsqueeze(1).transpose(-1, -2)).float() / math.sqrt(d)  # (B,H,T,n)
    s = s.masked_fill(~mask.unsqueeze(1), float("-inf"))
    if sink is not None:
        sk = sink.float().view(1, -1, 1, 1).expand(*s.shape[:-1], 1)
        p = torch.softmax(torch.cat([s, sk], -1), -1)[..., :-1]
    else:
        any_vis = mask.any(-1).unsqueeze(1).unsqueeze(-1)
        p = torch.softmax(torch.where(any_vis, s, torch.zeros_like(s)), -1)
        p = torch.where(any_vis, p, torch.zeros_like(p))
    return torch.matmul(p.to(kv.dtype), kv.unsqueeze(1))


@torch.no_grad()
def indexer_topk(idx: nn.Module, h: Tensor, is_visual: Tensor | None, chunk: int = 512) -> Tensor:
    """Lightning-indexer top-k block ids (B, T, k) with -1 for invalid picks."""
    b, t, _ = h.shape
    comp = idx.compressor
    y = lin.linear(h, torch.cat([_bf16(idx.w_dq.weight), _bf16(idx.w_w.weight), _bf16(comp.w_b_kv.weight),
                                 _bf16(comp.w_b_z.weight)], 0))
    c, nh = idx.c_indexer, idx.n_heads
    c_dq, w, cb, zb = torch.split(y, [c, nh, c, c], dim=-1)
    keys = _pool(cb, zb, comp.bias_b, comp.m)  # (B, n, c) fp32
    n_blocks = keys.shape[1]
    k_eff = min(idx.top_k, n_blocks)
    if k_eff == 0:
        return torch.full((b, t, 0), -1, dtype=torch.long, device=h.device)
    m_eff = t // n_blocks
    vis_bias = None
    if is_visual is not None:
        vis_bias = is_visual[:, : n_blocks * m_eff].reshape(b, n_blocks, m_eff).float().mean(-1)
    q = lin.linear(c_dq, idx.w_iuq.weight)  # (B, T, nh*c)
    keys_b = _bf16(keys)
    out = torch.empty(b, t, k_eff, dtype=torch.long, device=h.device)
    block_end = torch.arange(n_blocks, device=h.device) * m_eff + (m_eff - 1)
    for bi in range(b):
        for t0 in range(0, t, chunk):
            t1 = min(t, t0 + chunk)
            qc = q[bi, t0:t1].reshape((t1 - t0) * nh, c)
            s = gemm.gemm_nt(qc, keys_b[bi], out_dtype=torch.float32).view(t1 - t0, nh, n_blocks).clamp_(min=0.0)
            if vis_bias is not None:
                s += vis_bias[bi].view(1, 1, n_blocks) * 0.5
            sc = torch.einsum("thn,th->tn", s, w[bi, t0:t1].float())
            qpos = torch.arange(t0, t1, device=h.device).view(-1, 1)
            sc.masked_fill_(~(block_end.view(1, -1) < qpos), float("-inf"))
            vals, ids = sc.topk(k_eff, dim=-1)
            out[bi, t0:t1] = torch.where(torch.isfinite(vals), ids, torch.full_like(ids, -1))
    return out


def attention_forward(layer: nn.Module, kind: str, h: Tensor, is_visual: Tensor | None) -> Tensor:
    """Training/prefill forward (no KV cache) of SWA / CSA / HCA on CUDA."""
    from saint_llm_b200.models.attention.common import rope_tables

    cfg = layer.attn_cfg
    b, t, _ = h.shape
    H, d, rd = cfg.query_heads, cfg.head_dim, cfg.rope_dim
    hb = _bf16(h)
    ws = [layer.q_compressor.weight, layer.k_proj.weight, layer.v_proj.weight]
    sizes = [cfg.query_compression_dim, d, d]
    if kind != "swa":
        ws += [layer.kv_compressor.w_b_kv.weight, layer.kv_compressor.w_b_z.weight]
        sizes += [d, d]
    parts = torch.split(fused_linear(hb, ws), sizes, dim=-1)
    c_q, k, v = parts[0], parts[1], parts[2]
    cos, sin = rope_tables(t, rd, cfg.rope_theta, h.device)
    cos_b, sin_b = cos.repeat(b, 1), sin.repeat(b, 1)
    q = lin.linear(c_q, layer.q_up.weight).reshape(b * t, H, d)
    q = rope_norm(q, layer.q_norm.weight, cos_b, sin_b, rd, norm_first=False,
                  eps=layer.q_norm.eps).view(b, t, H, d).transpose(1, 2)
    k = rope_norm(k.reshape(b * t, 1, d), layer.k_norm.weight, cos_b, sin_b, rd,
                  norm_first=(kind == "csa"), eps=layer.k_norm.eps).view(b, t, d)
    v = v.contiguous()
    out = _sw_attention(q, k, v, cfg.sliding_window_size, layer.sink_logit, cfg.logit_softcap, layer)
    if kind in ("csa", "hca"):
        m = layer.csa_cfg.compression_rate if kind == "csa" else layer.hca_cfg.compression_rate
        comp = _pool(parts[3], parts[4], layer.kv_compressor.bias_b, m)
        n_blocks = comp.shape[1]
        if n_blocks > 0:
            kvn = rms_norm(_bf16(comp), layer.k_norm.weight, layer.k_norm.eps)
            if kind == "csa":
                top = indexer_topk(layer.indexer, hb, is_visual)
                if top.shape[-1] > 0:
                    sel = torch.zeros(b, t, n_blocks + 1, dtype=torch.bool, device=h.device)
                    sel.scatter_(2, torch.where(top >= 0, top, torch.full_like(top, n_blocks)), True)
                    out = out + _masked_compressed_attention(q, kvn, sel[..., :n_blocks], None).to(out.dtype)
            else:
                qpos = torch.arange(t, device=h.device).view(-1, 1)
                valid = (torch.arange(n_blocks, device=h.device).view(1, -1) * m + (m - 1) < qpos).unsqueeze(0)
                out = out + _masked_compressed_attention(q, kvn, valid, layer.sink_logit).to(out.dtype)
    flat = out.transpose(1, 2).reshape(b, t, H * d)
    return layer.output.forward_flat(flat)


__all__ = ["attention_forward", "fused_linear", "indexer_topk"]

"""CUDA training path of SWA / CSA / HCA attention.

Projections run on the native GEMM with the sibling projections of the same input
fused into one GEMM (``[q_compressor; k_proj; v_proj; w_b_kv; w_b_z]`` for attention,
``[w_dq; w_w; w_b_kv; w_b_z]`` for the indexer); Q/K RoPE+RMSNorm run as one fused
kernel per tensor in the reference's order (Q: rope then norm; K: CSA norm then rope,
SWA/HCA rope then norm).

The lightning indexer (no gradient flows through its integer output) is one fused
tcgen05 kernel (``csrc/indexer.cu``): scores = sum_h w_h relu(q_h . k_s) with the
strict block-causal mask, written once as (B, T, blocks); then top-k.

Attention itself is one fused tcgen05 kernel per direction (``csrc/attention.cu``): the
sliding-window branch (sink, softcap, max-logit telemetry) and the compressed branch
(HCA block-causal + sink, or CSA over the indexer's picks given as a bitmask -- exact,
because the top-k picks are a subset of the compressed table) run as two online
softmaxes whose outputs are summed; no score tensor ever reaches HBM.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.ops import backend, gemm
from saint_llm_b200.ops import linear as lin
from saint_llm_b200.ops.norm import rms_norm, rope_norm


def _bf16(t: Tensor) -> Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


class _FusedLinearFn(torch.autograd.Function):
    """y = x [W_0; W_1; ...]^T with per-weight gradients (into main_grad when present).

    ``fp8_owner`` (a module): the forward runs the block-scaled FP8 GEMM against the joint
    weight's FP8 copy cached on that module; the backward stays bf16 (straight-through)."""

    @staticmethod
    def forward(ctx, x: Tensor, fp8_owner: nn.Module | None, *weights: Tensor) -> Tensor:  # type: ignore[override]
        k = x.shape[-1]
        x2 = _bf16(x.reshape(-1, k))
        w = torch.cat([_bf16(wi) for wi in weights], 0)
        if fp8_owner is not None:
            from saint_llm_b200.ops import fp8

            y = fp8.gemm(fp8.quantize_rows(x2), fp8.cached_weight(fp8_owner, "_fp8_fused", list(weights)))
        else:
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
        return (dx, None, *grads)


def fused_linear(x: Tensor, weights: list[Tensor], fp8_owner: nn.Module | None = None) -> Tensor:
    return _FusedLinearFn.apply(x, fp8_owner, *weights)


def uses_fp8(linear: nn.Module) -> bool:
    """Whether a projection module runs the real block-scaled FP8 forward on CUDA."""
    return bool(getattr(linear, "use_real_fp8_gemm", False))


def _pool_torch(c_b: Tensor, z_b: Tensor, bias_b: Tensor, m: int) -> Tensor:
    """Softmax-over-m pooling (B, T, c) -> (B, T//m, c), fp32 math (CPU path and test oracle)."""
    b, t, c = c_b.shape
    n = t // m
    if n == 0:
        return c_b.new_zeros(b, 0, c, dtype=torch.float32)
    z = z_b[:, : n * m].float().reshape(b, n, m, c) + bias_b.float()
    return (torch.softmax(z, dim=-2) * c_b[:, : n * m].float().reshape(b, n, m, c)).sum(-2)


class _PoolFn(torch.autograd.Function):
    """``compress_pool_fwd`` / ``compress_pool_bwd`` (``csrc/pool.cu``): one kernel each way
    instead of the ~25 elementwise launches of the eager softmax pooling.  c_b / z_b are bf16
    column slices of the fused projection output; the bias gradient is the (b, s) sum of the
    kernel's fp32 dz."""

    @staticmethod
    def forward(ctx, c_b: Tensor, z_b: Tensor, bias_b: Tensor, m: int):  # type: ignore[override]
        b, t, c = c_b.shape
        out = torch.empty(b, t // m, c, dtype=torch.float32, device=c_b.device)
        backend.ext().compress_pool_fwd(c_b, z_b, bias_b.contiguous(), m, out)
        ctx.save_for_backward(c_b, z_b, bias_b, out)
        ctx.m = m
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        c_b, z_b, bias_b, out = ctx.saved_tensors
        m = ctx.m
        b, t, c = c_b.shape
        n = t // m
        if n * m == t:
            dc = torch.empty(b, t, c, dtype=c_b.dtype, device=c_b.device)
            dz = torch.empty_like(dc)
        else:
            dc = torch.zeros(b, t, c, dtype=c_b.dtype, device=c_b.device)
            dz = torch.zeros_like(dc)
        dz32 = torch.empty(b, n, m, c, dtype=torch.float32, device=c_b.device)
        backend.ext().compress_pool_bwd(c_b, z_b, bias_b.contiguous(), m, out, dout.float().contiguous(), dc, dz,
                                        dz32)
        dbias = dz32.sum((0, 1)).to(bias_b.dtype)
        return dc, dz, dbias, None


def _pool(c_b: Tensor, z_b: Tensor, bias_b: Tensor, m: int) -> Tensor:
    """Softmax-over-m pooling (B, T, c) -> (B, T//m, c) fp32 (reference
    core/attention/csa.py TokenLevelCompressor): the fused kernel on CUDA for bf16 inputs."""
    b, t, c = c_b.shape
    if (c_b.is_cuda and c_b.dtype == torch.bfloat16 and z_b.dtype == torch.bfloat16 and t // m > 0
            and c_b.stride(-1) == 1 and z_b.stride(-1) == 1 and c_b.stride(0) == t * c_b.stride(1)
            and z_b.stride(0) == t * z_b.stride(1)):
        return _PoolFn.apply(c_b, z_b, bias_b, m)
    return _pool_torch(c_b, z_b, bias_b, m)


def _pad_head(t: Tensor, hd: int) -> Tensor:
    return t if t.shape[-1] == hd else F.pad(t, (0, hd - t.shape[-1]))


class _FusedAttnFn(torch.autograd.Function):
    """Window branch (+ sink, softcap) and optional compressed branch in one tcgen05 kernel.

    q (B, T, H, d), k/v (B, T, d), kv (B, n, d) (K = V, already k-normed), sink (H) or None,
    sel: CSA selection bits (B, T, words) or None.  Returns (B, T, H, d) = o_window + o_comp.
    """

    @staticmethod
    def forward(ctx, q, k, v, kv, sink, sel, mode, m, window, softcap, maxlogit):  # type: ignore[override]
        d = q.shape[-1]
        hd = 64 if d <= 64 else 128
        if d > 128:
            raise ValueError("fused attention supports head_dim <= 128")
        qb, kb_, vb = (_pad_head(_bf16(t), hd).contiguous() for t in (q, k, v))
        kvb = _pad_head(_bf16(kv), hd).contiguous() if mode else qb.new_empty(0)
        b, t, h = q.shape[:3]
        ext = backend.ext()
        o_sw = torch.empty(b, t, h, hd, dtype=torch.bfloat16, device=q.device)
        o_c = torch.empty_like(o_sw) if mode else o_sw.new_empty(0)
        out = torch.empty_like(o_sw) if mode else o_sw
        lse = torch.empty(2, b, h, t, dtype=torch.float32, device=q.device)
        sink_f = sink.float().contiguous() if sink is not None else lse.new_empty(0)
        sel_t = sel if sel is not None else torch.empty(0, dtype=torch.int32, device=q.device)
        # the kernel max-reduces |logit| into an fp32 scalar
        ml = None
        if maxlogit is not None:
            ml = maxlogit if maxlogit.dtype == torch.float32 and maxlogit.numel() == 1 else \
                torch.zeros((), dtype=torch.float32, device=q.device)
            ml.zero_()
        ext.attn_fwd(qb, kb_, vb, kvb, sel_t, mode, m, window, sink_f, float(softcap or 0.0), 1.0 / math.sqrt(d),
                     o_sw, o_c, out, lse, ml if ml is not None else lse.new_empty(0), gemm.error_word(q.device))
        if ml is not None and ml is not maxlogit:
            maxlogit.copy_(ml)
        ctx.save_for_backward(qb, kb_, vb, kvb, sink_f, sel_t, o_sw, o_c, lse)
        ctx.meta = (mode, m, window, float(softcap or 0.0), d, sink is not None,
                    sink.dtype if sink is not None else None, kv.dtype if mode else None)
        return out[..., :d]

    @staticmethod
    def backward(ctx, dout):  # type: ignore[override]
        qb, kb_, vb, kvb, sink_f, sel_t, o_sw, o_c, lse = ctx.saved_tensors
        mode, m, window, softcap, d, has_sink, sink_dtype, kv_dtype = ctx.meta
        hd = qb.shape[-1]
        dob = _pad_head(_bf16(dout), hd).contiguous()
        dq = torch.empty_like(qb)
        dk = torch.zeros(kb_.shape, dtype=torch.float32, device=qb.device)
        dv = torch.zeros_like(dk)
        dkv = torch.zeros(kvb.shape, dtype=torch.float32, device=qb.device) if mode else dk.new_empty(0)
        dsink = torch.zeros_like(sink_f)
        backend.ext().attn_bwd(qb, kb_, vb, kvb, sel_t, mode, m, window, sink_f, softcap, 1.0 / math.sqrt(d), o_sw,
                               o_c, lse, dob, dq, dk, dv, dkv, dsink, gemm.error_word(qb.device))
        gkv = dkv[..., :d].to(kv_dtype) if mode else None
        gs = dsink.to(sink_dtype) if has_sink else None
        return (dq[..., :d], dk[..., :d].to(torch.bfloat16), dv[..., :d].to(torch.bfloat16), gkv, gs,
                None, None, None, None, None, None)


def fused_attention(q: Tensor, k: Tensor, v: Tensor, *, window: int, sink: Tensor | None, softcap: float | None,
                    kv: Tensor | None = None, mode: int = 0, m: int = 1, sel: Tensor | None = None,
                    maxlogit: Tensor | None = None) -> Tensor:
    """Sliding-window attention (+ compressed branch) on the native kernel; see ``_FusedAttnFn``."""
    if mode and (kv is None or kv.shape[1] == 0):
        mode, kv = 0, None
    return _FusedAttnFn.apply(q, k, v, kv if mode else q.new_empty(0), sink, sel, mode, m, window, softcap, maxlogit)


@torch.no_grad()
def _indexer_scores(idx: nn.Module, h: Tensor, is_visual: Tensor | None) -> tuple[Tensor | None, int, int]:
    """(scores (B, T, blocks) with -inf where block-causally masked, k_eff, n_blocks) from
    the fused ``indexer_scores`` kernel (one pass; only the (B, T, blocks) scores are
    written).  scores is None when no block exists yet."""
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
        return None, 0, n_blocks
    m_eff = t // n_blocks
    vis_bias = None
    if is_visual is not None:
        vis_bias = is_visual[:, : n_blocks * m_eff].reshape(b, n_blocks, m_eff).float().mean(-1)
    q = lin.linear(c_dq, idx.w_iuq.weight)  # (B, T, nh*c)
    keys_b = _bf16(keys)
    cp = 64 if c <= 64 else 128
    if c > 128:
        raise ValueError("indexer head dim above 128 is not supported by the fused indexer kernel")
    if cp != c:  # zero-padding the head dim leaves every dot product unchanged
        q = F.pad(q.view(b, t, nh, c), (0, cp - c)).view(b, t, nh * cp)
        keys_b = F.pad(keys_b, (0, cp - c))
    scores = torch.empty(b, t, n_blocks, dtype=torch.float32, device=h.device)
    backend.ext().indexer_scores(q.contiguous(), keys_b.contiguous(), w.float().contiguous(),
                                 None if vis_bias is None else vis_bias.contiguous(), m_eff, 0, scores,
                                 gemm.error_word(h.device))
    return scores, k_eff, n_blocks


def indexer_topk(idx: nn.Module, h: Tensor, is_visual: Tensor | None) -> Tensor:
    """Lightning-indexer top-k block ids (B, T, k) with -1 for invalid picks."""
    b, t, _ = h.shape
    scores, k_eff, _ = _indexer_scores(idx, h, is_visual)
    if scores is None:
        return torch.full((b, t, 0), -1, dtype=torch.long, device=h.device)
    vals, ids = scores.topk(k_eff, dim=-1)
    return torch.where(torch.isfinite(vals), ids, torch.full_like(ids, -1))


def indexer_select(idx: nn.Module, h: Tensor, is_visual: Tensor | None) -> Tensor | None:
    """The CSA selection bitmask (B, T, ceil(blocks / 32)) int32 of the indexer's top-k
    finite blocks per query, straight from the scores by one native kernel (radix selection
    of the k-th score; ties at it taken lowest block index first); None when no block exists."""
    b, t, _ = h.shape
    scores, k_eff, n_blocks = _indexer_scores(idx, h, is_visual)
    if scores is None:
        return None
    sel = torch.empty(b, t, (n_blocks + 31) // 32, dtype=torch.int32, device=h.device)
    backend.ext().indexer_select_mask(scores, k_eff, sel)
    return sel


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
    fp8_proj = uses_fp8(layer.q_compressor) and all(w.shape[0] % 128 == 0 for w in ws) and hb.shape[-1] % 128 == 0
    parts = torch.split(fused_linear(hb, ws, layer if fp8_proj else None), sizes, dim=-1)
    c_q, k, v = parts[0], parts[1], parts[2]
    cos, sin = rope_tables(t, rd, cfg.rope_theta, h.device)
    cos_b, sin_b = cos.repeat(b, 1), sin.repeat(b, 1)
    if uses_fp8(layer.q_up) and lin.fp8_shape_ok(layer.q_up.in_features, layer.q_up.out_features):
        q = lin.fp8_linear(c_q, layer.q_up.weight).reshape(b * t, H, d)
    else:
        q = lin.linear(c_q, layer.q_up.weight).reshape(b * t, H, d)
    q = rope_norm(q, layer.q_norm.weight, cos_b, sin_b, rd, norm_first=False, eps=layer.q_norm.eps)
    k = rope_norm(k.reshape(b * t, 1, d), layer.k_norm.weight, cos_b, sin_b, rd,
                  norm_first=(kind == "csa"), eps=layer.k_norm.eps).view(b, t, d)
    q = q.view(b, t, H, d)
    mode, m, kvn, sel = 0, 1, None, None
    if kind in ("csa", "hca"):
        m = layer.csa_cfg.compression_rate if kind == "csa" else layer.hca_cfg.compression_rate
        comp = _pool(parts[3], parts[4], layer.kv_compressor.bias_b, m)
        n_blocks = comp.shape[1]
        if n_blocks > 0:
            kvn = rms_norm(_bf16(comp), layer.k_norm.weight, layer.k_norm.eps)
            if kind == "csa":
                sel = indexer_select(layer.indexer, hb, is_visual)
                if sel is not None:
                    mode = 2
            else:
                mode = 1
    out = fused_attention(q, k, v.contiguous(), window=cfg.sliding_window_size, sink=layer.sink_logit,
                          softcap=cfg.logit_softcap, kv=kvn, mode=mode, m=m, sel=sel,
                          maxlogit=layer.max_attn_logit)
    flat = out.reshape(b, t, H * d)
    return layer.output.forward_flat(flat)


__all__ = ["attention_forward", "fused_linear", "indexer_select", "indexer_topk"]

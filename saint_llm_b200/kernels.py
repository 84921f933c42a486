"""Kernel-level public functions under the names a user of the reference's kernels package
calls (``saint_llm_kernels/__init__.py``), backed by this framework's sm_100a kernels.

Each ``*_reference`` function is the plain fp32 PyTorch definition of the operation (the
oracle the tests compare against); the function without the suffix runs the native kernel on
a B200 with the extension built and the same definition elsewhere:

* ``lightning_indexer_scores`` / ``_topk``: the fused tcgen05 indexer kernel
  (``csrc/indexer.cu``: head-weighted ReLU scores reduced in registers, only the
  (B, T, n_blocks) scores are written; reference ``kernels/attention.py:33-128``);
* ``mhc_carry``: the fused mHC combine ``B X + C (x) out`` (``csrc/norm.cu`` ``mhc_combine``,
  with its backward; reference ``kernels/mhc.py:32-70``);
* ``fp8_gemm``: the block-scaled FP8 GEMM (1 x 128 activation blocks, 128 x 128 weight blocks,
  ``kind::mxf8f6f4.block_scale``; reference ``kernels/fp8_gemm.py:86-103``, which scales per
  row / per output channel) with a straight-through backward.

The quantisation helpers, the FP8 / FP4 linears and the grouped expert GEMM are re-exported
from where they live (``ops.quant``, ``models.linear``, ``ops.moe``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from saint_llm_b200.models.linear import Fp4Linear, Fp8Linear
from saint_llm_b200.ops import backend
from saint_llm_b200.ops.moe import GroupedSwiGLUExperts, grouped_mm
from saint_llm_b200.ops.quant import (
    Fp8Format,
    cast_to_fp4_mx,
    cast_to_fp8,
    dequant_from_fp4_mx,
    dequant_from_fp8,
    fake_quant_fp4_mx,
    fake_quant_fp8,
)


def _native(t: Tensor) -> bool:
    return t.is_cuda and backend.native_for(t)


# ------------------------------------------------------------------ lightning indexer
def lightning_indexer_scores_reference(q_indexer: Tensor, k_compressed: Tensor, head_weights: Tensor,
                                       visual_bias: Tensor | None = None) -> Tensor:
    """(B, T, n_blocks) unmasked scores: sum_h w[b,t,h] * (ReLU(q[b,t,h] . k[b,s]) + 0.5 vis[b,s]).

    q_indexer (B, T, H, c); k_compressed (B, n_blocks, c); head_weights (B, T, H);
    visual_bias (B, n_blocks) or None."""
    s = torch.einsum("bthc,bnc->bthn", q_indexer.float(), k_compressed.float()).clamp(min=0.0)
    if visual_bias is not None:
        s = s + 0.5 * visual_bias.float()[:, None, None, :]
    return (head_weights.float().unsqueeze(-1) * s).sum(2)


def _block_visible(t: int, n_blocks: int, m: int, device: torch.device) -> Tensor:
    """visible[q, s]: block s (tokens s*m .. s*m + m - 1) is complete strictly before query q."""
    end = torch.arange(n_blocks, device=device) * m + (m - 1)
    return end[None, :] < torch.arange(t, device=device)[:, None]


def _topk_ids(masked: Tensor, top_k: int) -> Tensor:
    vals, ids = masked.topk(min(top_k, masked.shape[-1]), dim=-1)
    return torch.where(torch.isfinite(vals), ids, torch.full_like(ids, -1))


def lightning_indexer_topk_reference(q_indexer: Tensor, k_compressed: Tensor, head_weights: Tensor, top_k: int,
                                     block_size_m: int, visual_bias: Tensor | None = None) -> Tensor:
    """(B, T, min(top_k, n_blocks)) ids of the best-scoring complete blocks per query; -1 where
    fewer blocks are visible; (B, T, 0) when there is no block or ``top_k`` is 0."""
    b, t = q_indexer.shape[:2]
    nb = k_compressed.shape[1]
    if top_k == 0 or nb == 0:
        return torch.full((b, t, 0), -1, dtype=torch.long, device=q_indexer.device)
    s = lightning_indexer_scores_reference(q_indexer, k_compressed, head_weights, visual_bias)
    vis = _block_visible(t, nb, block_size_m, q_indexer.device)
    return _topk_ids(s.masked_fill(~vis, float("-inf")), top_k)


def _native_scores(q: Tensor, k: Tensor, w: Tensor, vis: Tensor | None, m: int, q_start: int) -> Tensor:
    """The indexer kernel: block n is kept iff n*m + m - 1 < q_start + t, else -inf."""
    from saint_llm_b200.ops import gemm

    b, t, nh, c = q.shape
    nb = k.shape[1]
    cp = 64 if c <= 64 else 128
    if c > 128:
        raise ValueError("the fused indexer kernel takes head dims up to 128")
    qb = F.pad(q.to(torch.bfloat16), (0, cp - c)).reshape(b, t, nh * cp).contiguous()
    kb = F.pad(k.to(torch.bfloat16), (0, cp - c)).contiguous()  # zero padding keeps every dot product
    out = torch.empty(b, t, nb, dtype=torch.float32, device=q.device)
    backend.ext().indexer_scores(qb, kb, w.float().contiguous(), None if vis is None else vis.float().contiguous(),
                                 m, q_start, out, gemm.error_word(q.device))
    return out


def lightning_indexer_scores(q_indexer: Tensor, k_compressed: Tensor, head_weights: Tensor,
                             visual_bias: Tensor | None = None) -> Tensor:
    """``lightning_indexer_scores_reference`` on the fused kernel (bf16 operands, fp32 scores)."""
    if not _native(q_indexer) or k_compressed.shape[1] == 0:
        return lightning_indexer_scores_reference(q_indexer, k_compressed, head_weights, visual_bias)
    # with block size 1 and queries starting at n_blocks every block counts as complete
    return _native_scores(q_indexer, k_compressed, head_weights, visual_bias, 1, k_compressed.shape[1])


def lightning_indexer_topk(q_indexer: Tensor, k_compressed: Tensor, head_weights: Tensor, top_k: int,
                           block_size_m: int, visual_bias: Tensor | None = None) -> Tensor:
    """``lightning_indexer_topk_reference`` with the block-causal scores from the fused kernel."""
    nb = k_compressed.shape[1]
    if not _native(q_indexer) or top_k == 0 or nb == 0:
        return lightning_indexer_topk_reference(q_indexer, k_compressed, head_weights, top_k, block_size_m,
                                                visual_bias)
    return _topk_ids(_native_scores(q_indexer, k_compressed, head_weights, visual_bias, block_size_m, 0), top_k)


# ----------------------------------------------------------------------------- mHC
def mhc_carry_reference(b_l: Tensor, c_l: Tensor, x: Tensor, inner_out: Tensor) -> Tensor:
    """out[b,t,h] = sum_k b_l[b,t,h,k] x[b,t,k] + c_l[b,t,h] inner_out[b,t]: (B, T, n_hc, d)."""
    return torch.einsum("bthk,btkd->bthd", b_l, x) + c_l.unsqueeze(-1) * inner_out.unsqueeze(2)


def mhc_carry(b_l: Tensor, c_l: Tensor, x: Tensor, inner_out: Tensor) -> Tensor:
    """``mhc_carry_reference`` as one fused kernel (bf16 streams, fp32 gates; differentiable)."""
    if not _native(x):
        return mhc_carry_reference(b_l, c_l, x, inner_out)
    from saint_llm_b200.ops.mhc import mhc_combine

    return mhc_combine(x, inner_out, b_l, c_l).to(x.dtype)


# ----------------------------------------------------------------------------- FP8
def is_fp8_gemm_supported(device: torch.device | None = None) -> bool:
    """True where ``fp8_gemm`` runs the block-scaled tensor-core kernel: a B200 (sm_100)
    with this framework's extension loaded."""
    if device is None:
        if not torch.cuda.is_available():
            return False
        device = torch.device("cuda")
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        return False
    try:
        backend.ext()
    except Exception:  # noqa: BLE001 - not built: no native FP8 GEMM
        return False
    return True


class _Fp8GemmFn(torch.autograd.Function):
    """Forward: activations quantised per 1 x 128 block, the weight per 128 x 128 block (fresh
    every call: no cached copy can go stale); backward: straight-through, in the weight dtype."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, out_dtype: torch.dtype) -> Tensor:  # type: ignore[override]
        from saint_llm_b200.ops import fp8

        ctx.save_for_backward(x, weight)
        return fp8.linear(x, weight).to(out_dtype)

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x, weight = ctx.saved_tensors
        k = weight.shape[1]
        dy2 = dy.reshape(-1, weight.shape[0]).to(weight.dtype)
        dx = (dy2 @ weight).reshape(x.shape).to(x.dtype)
        dw = (dy2.t() @ x.reshape(-1, k).to(weight.dtype)) if ctx.needs_input_grad[1] else None
        return dx, dw, None


def fp8_gemm(x: Tensor, weight: Tensor, *, weight_fmt: Fp8Format = Fp8Format.E4M3,
             activation_fmt: Fp8Format = Fp8Format.E4M3, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """``x @ weight^T`` through block-scaled E4M3 FP8 (x (..., K), weight (N, K), K and N
    multiples of 128) with a straight-through backward.  On a device without the native
    kernel (``is_fp8_gemm_supported`` False) the same quantisation runs as a dequantised
    matmul, so the numbers agree with the kernel's."""
    if weight_fmt is not Fp8Format.E4M3 or activation_fmt is not Fp8Format.E4M3:
        raise ValueError("the block-scaled FP8 GEMM takes E4M3 operands")
    n, k = weight.shape
    if x.shape[-1] != k:
        raise ValueError(f"K mismatch: x (..., {x.shape[-1]}) vs weight ({n}, {k})")
    if k % 128 or n % 128:
        raise ValueError(f"the block-scaled FP8 GEMM needs K and N divisible by 128; got K={k}, N={n}")
    return _Fp8GemmFn.apply(x, weight, out_dtype)


__all__ = [
    "Fp4Linear",
    "Fp8Format",
    "Fp8Linear",
    "GroupedSwiGLUExperts",
    "cast_to_fp4_mx",
    "cast_to_fp8",
    "dequant_from_fp4_mx",
    "dequant_from_fp8",
    "fake_quant_fp4_mx",
    "fake_quant_fp8",
    "fp8_gemm",
    "grouped_mm",
    "is_fp8_gemm_supported",
    "lightning_indexer_scores",
    "lightning_indexer_scores_reference",
    "lightning_indexer_topk",
    "lightning_indexer_topk_reference",
    "mhc_carry",
    "mhc_carry_reference",
]

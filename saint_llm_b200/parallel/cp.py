"""Two-stage context parallelism for the CSA / HCA / SWA / NSA stack (absent in the
reference; planned there).  The sequence is split into contiguous shards, rank r of a
CP group of size c holds tokens ``[r*Tl, (r+1)*Tl)``; everything except attention is
per token, so only attention exchanges data:

* stage 1 — compressed entries: each rank compresses its own blocks (shards are
  block-aligned) and the entries of all ranks are all-gathered (HCA's dense compressed
  branch, CSA's top-k sparse branch and its lightning-indexer keys all index global
  block numbers); the all-gather's backward sums the gradients back to their owners;
* stage 2 — the sliding-window halo: the last ``w`` post-RoPE K/V rows of rank r-1
  reach rank r, and their gradients travel back.

Both stages share one all-gather per layer (tails and compressed entries packed in one
buffer; with one MQA K/V head a tail is ``w x 2 x head_dim`` values), so every rank
issues the same collectives in the same order in forward and backward — two separate
exchanges per layer could be reordered by the autograd engine on one rank and not on
another.

The attention modules are run unchanged through their KV-cache entry point: a
``CPLayerView`` presents "the context before this shard" exactly as a cache would
(``length`` = the shard's start, so RoPE and every block-causal / window mask use
global positions).  For SWA / CSA / HCA layers the window K/V are only the halo and the
local rows, with ``key_offset`` = the global position of the first halo row (the window
branch reads keys from there), so no rank holds K/V for the whole sequence.  NSA, whose
compressed and selective branches index keys from position 0, gets the keys at full length
with zeros before the halo (outside every query's window, so never attended).
"""

from __future__ import annotations

import contextlib
from collections.abc import Iterator

import torch
import torch.distributed as dist
from torch import Tensor, nn


class _GatherStack(torch.autograd.Function):
    """(ws, *x.shape) = every rank's ``x``; the backward sums the gradient over ranks and
    keeps this rank's slice."""

    @staticmethod
    def forward(ctx, x: Tensor, group: object) -> Tensor:  # type: ignore[override]
        ctx.group = group
        parts = [torch.empty_like(x) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.stack(parts)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g[dist.get_rank(ctx.group)], None


def gather_stack(x: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    return _GatherStack.apply(x, group)


class CPLayerView:
    """Cache-shaped view of the context before this rank's shard, for one layer.

    One collective per layer and direction: every rank contributes its window tail
    (the last ``w`` K/V rows) and its compressed entries packed in one buffer; the
    all-gather gives each rank the previous rank's tail (the halo) and every rank's
    compressed entries in global block order."""

    # CSA asks for the gathered per-block visual fractions (the indexer's cohesion bias) through
    # ``append(..., is_visual=...)``; decode caches, which the reference leaves without it, do not
    carries_visual_bias = True

    def __init__(self, group: dist.ProcessGroup | None, shard_len: int, window: int, *, compact: bool = True) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.ws = dist.get_world_size(group)
        self.length = self.rank * shard_len
        self.window = min(window, shard_len)
        self.compact = compact
        self.key_offset = 0

    def append(self, *args: Tensor, compressor=None, indexer_compressor=None,  # noqa: ANN001, ANN201
               is_visual: Tensor | None = None):
        if compressor is None:  # SWA / NSA: (k, v)
            h, (k, v) = None, args
        else:
            h, k, v = args
        b, d, w = k.shape[0], k.shape[-1], self.window
        parts = [torch.cat([k[:, -w:], v[:, -w:]], -1)]
        visual = compressor is not None and indexer_compressor is not None and is_visual is not None
        if compressor is not None:
            parts.append(compressor(h))
            if indexer_compressor is not None:
                # the indexer's keys only choose blocks (top-k has no gradient); without the
                # no-grad they would still receive zeros through the packed gather and the
                # optimizer would decay weights the unsharded model leaves untouched
                with torch.no_grad():
                    parts.append(indexer_compressor(h))
            if visual:  # the fraction of image tokens per local block, gathered with the entries
                m = indexer_compressor.m
                nb = h.shape[1] // m
                parts.append(is_visual[:, :nb * m].reshape(b, nb, m).to(h.dtype).mean(-1, keepdim=True))
        sizes = [p.shape[1:] for p in parts]
        g = gather_stack(torch.cat([p.reshape(b, -1) for p in parts], 1), self.group)  # (ws, B, L)
        outs, off = [], 0
        for shp in sizes:
            n = shp.numel()
            outs.append(g[:, :, off:off + n].reshape(self.ws, b, *shp))
            off += n
        if self.rank == 0:  # no halo; the empty slice keeps the gather in the graph on every rank
            empty = outs[0][0][:, :0]
            k_all, v_all = torch.cat([empty[..., :d], k], 1), torch.cat([empty[..., d:], v], 1)
        elif self.compact:  # halo + local rows; the window branch starts at key_offset
            halo = outs[0][self.rank - 1]
            self.key_offset = self.length - w
            k_all = torch.cat([halo[..., :d], k], 1)
            v_all = torch.cat([halo[..., d:], v], 1)
        else:
            halo = outs[0][self.rank - 1]
            z = k.new_zeros(b, self.length - w, d)
            k_all = torch.cat([z, halo[..., :d], k], 1)
            v_all = torch.cat([z, halo[..., d:], v], 1)
        if compressor is None:
            return k_all, v_all
        comp = [o.transpose(0, 1).reshape(b, -1, o.shape[-1]) for o in outs[1:]]
        if indexer_compressor is None:  # HCA
            return comp[0], k_all, v_all
        if visual:
            return comp[0], comp[1], k_all, v_all, comp[2].squeeze(-1)
        return comp[0], comp[1], k_all, v_all


class CPBundle:
    """Per-layer CP views for ``model.backbone(..., kv_cache_bundle=CPBundle(...))``."""

    def __init__(self, model: nn.Module, group: dist.ProcessGroup | None, shard_len: int) -> None:
        cfg = model.cfg  # type: ignore[attr-defined]
        if cfg.n_sink_tokens:
            raise ValueError("context parallelism does not support prepended sink tokens")
        rates = {"csa": cfg.csa.compression_rate, "hca": cfg.hca.compression_rate, "nsa": cfg.nsa.compression_rate}
        kinds = {cfg.layer_kind(i) for i in range(len(model.blocks))}  # type: ignore[arg-type]
        for m in (rates[k] for k in kinds if k in rates):
            if shard_len % m:
                raise ValueError(f"shard length {shard_len} must be a multiple of every compression rate ({m})")
        if shard_len < cfg.attention.sliding_window_size:
            raise ValueError("shard length must be at least the sliding window")
        self.views = [CPLayerView(group, shard_len, cfg.attention.sliding_window_size,
                                  compact=cfg.layer_kind(i) != "nsa")
                      for i in range(len(model.blocks))]  # type: ignore[arg-type]
        self.length = self.views[0].length

    def for_layer(self, i: int) -> CPLayerView:
        return self.views[i]


@contextlib.contextmanager
def balance_over(model: nn.Module, group: dist.ProcessGroup | None) -> Iterator[None]:
    """While active, every MoE layer of ``model`` computes its balance loss over sequences
    sharded across ``group`` (``models.moe.sharded_balance_loss``): the loss's per-sequence
    statistics span every shard."""
    layers = [m for m in model.modules() if hasattr(m, "balance_group")]
    for m in layers:
        m.balance_group = group if group is not None else dist.group.WORLD  # None would mean "off"
    try:
        yield
    finally:
        for m in layers:
            m.balance_group = None


def cp_shard(ids: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    """This rank's contiguous slice of (B, T) token ids."""
    r, ws = dist.get_rank(group), dist.get_world_size(group)
    t = ids.shape[1] // ws
    return ids[:, r * t:(r + 1) * t]


def _ce_share(model: nn.Module, h: Tensor, ids: Tensor, start: int, shift: int) -> Tensor:
    """Sum of CE(logits(h[:, j]), ids[:, start + j + shift]) over the local positions j whose
    target exists, divided by the global count B * (T - shift): this shard's share of the
    mean next-``shift``-token loss."""
    b, t = ids.shape
    n = max(0, min(h.shape[1], t - shift - start))
    if n == 0:
        return h.sum() * 0.0  # keeps the graph (and the CP collectives' backward) on every rank
    logits = model.logits(h[:, :n]).float()  # type: ignore[attr-defined]
    tgt = ids[:, start + shift:start + shift + n]
    ce = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1), reduction="sum")
    return ce / (b * (t - shift))


def cp_lm_loss(model: nn.Module, ids: Tensor, group: dist.ProcessGroup | None = None, *,
               mtp: bool = False, balance: bool = False) -> Tensor:
    """Next-token cross-entropy of the full sequence ``ids`` (B, T) computed with its tokens
    sharded over ``group``; returns this rank's share of the global mean (the sum over
    ranks is the loss).

    ``mtp``: add the multi-token-prediction heads' weighted losses (the training loss of
    ``train.losses.cross_entropy_with_mtp`` without the balance term).  Head k combines the
    hidden state at position p with the embedding of token p + k + 1, which for a shard's
    last positions lies in the next shard: every rank holds all token ids, so it embeds the
    few it needs itself and the heads need no communication.

    ``balance``: add ``sequence_balance_weight`` x the MoE balance loss, computed over the whole
    sequences (``balance_over``): with ``mtp`` too, the sum over ranks is the training loss of
    ``cross_entropy_with_mtp`` with its balance term."""
    r, ws = dist.get_rank(group), dist.get_world_size(group)
    tl = ids.shape[1] // ws
    start = r * tl
    local = ids[:, start:start + tl]
    with balance_over(model, group):
        h, _ = model.backbone(local, kv_cache_bundle=CPBundle(model, group, tl))  # type: ignore[attr-defined]
    loss = shard_loss(model, h, ids, start, mtp=mtp)
    w = model.cfg.moe.sequence_balance_weight if balance else 0.0  # type: ignore[attr-defined]
    aux = model.aux_loss() if w else None  # type: ignore[attr-defined]
    return loss + w * aux if aux is not None else loss


def shard_loss(model: nn.Module, h: Tensor, ids: Tensor, start: int, *, mtp: bool = False) -> Tensor:
    """This shard's share of the training loss from its final-normed hidden states ``h``
    (positions ``start ..``) and the full token ids: main next-token CE, plus (``mtp``) the
    MTP heads' weighted CEs.  Summed over the shards it is the loss of the whole sequence."""
    b, t = ids.shape
    tl = h.shape[1]
    loss = _ce_share(model, h, ids, start, 1)
    depth = model.cfg.mtp.depth if mtp else 0  # type: ignore[attr-defined]
    if depth > 0:
        from saint_llm_b200.train.losses import mtp_weight

        ahead = ids[:, start:min(t, start + tl + depth)]
        emb = model._embed_inputs(ahead, None, None)  # type: ignore[attr-defined]
        emb = torch.nn.functional.pad(emb, (0, 0, 0, tl + depth - emb.shape[1]))  # zeros past the end
        cur = h
        for k, mod in enumerate(model.mtp.modules_):  # type: ignore[attr-defined]
            cur = mod(cur, emb[:, k + 1:k + 1 + tl])
            loss = loss + mtp_weight(model.cfg.mtp, k) * _ce_share(model, cur, ids, start, k + 2)  # type: ignore[attr-defined]
    return loss


__all__ = ["CPBundle", "CPLayerView", "balance_over", "cp_lm_loss", "cp_shard", "gather_stack", "shard_loss"]

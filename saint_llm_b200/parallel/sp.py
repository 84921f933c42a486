"""Sequence parallelism for dense / sliding-window attention: Ulysses all-to-all, ring
attention, and zigzag sharding (all absent in the reference, planned there for v0.4 --
``docs/ROADMAP.md:307``; the V4 stack's own long-context path is the two-stage context
parallelism of ``parallel.cp``, these are the generic sequence-parallel forms).

Tensors are (B, T_local, H, d) shards of a (B, T, H, d) sequence.  Positions are explicit
(``q_pos`` / ``k_pos``, global token indices of the local rows), so the masks stay right under
any sharding -- contiguous (rank r holds block r) or zigzag (rank r holds blocks r and
2P-1-r of 2P, which balances causal work across ranks).

* ``ulysses_attention``: an all-to-all turns sequence shards into head shards (every rank
  gets the whole sequence for H / P heads), attention runs locally, a second all-to-all
  turns the result back.  Communication: 4 all-to-alls of the local activations.
* ``ring_attention``: K / V shards travel around the ring (P - 1 hops); each rank merges
  the partial softmax of every block with a running log-sum-exp, skipping the math of
  blocks the mask hides completely.  Each hop completes before the next block's math (no
  overlap yet).

Both are differentiable: the all-to-all's backward is the inverse all-to-all, the ring hop's
backward sends the gradient the opposite way.  Point-to-point exchanges use grouped
``batch_isend_irecv`` (gloo has no all-to-all), posted identically on every rank.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor


def _a2a(parts: list[Tensor], group: dist.ProcessGroup | None) -> list[Tensor]:
    """out[j] = rank j's parts[my rank] (all parts of one rank have equal shapes per peer)."""
    rank, ws = dist.get_rank(group), dist.get_world_size(group)
    out = [torch.empty(parts[rank].shape, dtype=parts[rank].dtype, device=parts[rank].device) for _ in range(ws)]
    out[rank] = parts[rank].contiguous()
    ops = []
    for j in range(ws):
        if j == rank:
            continue
        peer = dist.get_global_rank(group, j) if group is not None else j
        ops.append(dist.P2POp(dist.isend, parts[j].contiguous(), peer, group))
        ops.append(dist.P2POp(dist.irecv, out[j], peer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return out


class _SeqToHead(torch.autograd.Function):
    """(B, T_local, H, d) sequence shard -> (B, T, H / P, d) head shard (rank order along T)."""

    @staticmethod
    def forward(ctx, x: Tensor, group):  # type: ignore[override]
        ctx.group = group
        ws = dist.get_world_size(group)
        parts = list(x.chunk(ws, dim=2))
        return torch.cat(_a2a(parts, group), dim=1)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return _HeadToSeq.apply(g, ctx.group), None


class _HeadToSeq(torch.autograd.Function):
    """Inverse of ``_SeqToHead``."""

    @staticmethod
    def forward(ctx, x: Tensor, group):  # type: ignore[override]
        ctx.group = group
        ws = dist.get_world_size(group)
        parts = list(x.chunk(ws, dim=1))
        return torch.cat(_a2a(parts, group), dim=2)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return _SeqToHead.apply(g, ctx.group), None


def _block(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, k_pos: Tensor, causal: bool, window: int | None,
           scale: float) -> tuple[Tensor, Tensor]:
    """Partial attention of q (B, Tq, H, d) over one K/V block: (out, lse) with out
    normalised within the block; rows with no visible key get lse = -inf and out = 0."""
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) * scale
    vis = torch.ones(q_pos.numel(), k_pos.numel(), dtype=torch.bool, device=q.device)
    if causal:
        vis &= k_pos[None, :] <= q_pos[:, None]
    if window is not None:
        vis &= k_pos[None, :] > q_pos[:, None] - window
    s = s.masked_fill(~vis, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                               # (B, H, Tq)
    safe = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    p = torch.exp(s - safe[..., None])
    out = torch.einsum("bhqk,bkhd->bqhd", p, v.float())
    return out, lse


def local_attention(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, k_pos: Tensor, *, causal: bool = True,
                    window: int | None = None) -> Tensor:
    """Reference attention on one process (fp32 math, output in q's dtype)."""
    out, _ = _block(q, k, v, q_pos, k_pos, causal, window, 1.0 / math.sqrt(q.shape[-1]))
    return out.to(q.dtype)


def ulysses_attention(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, group: dist.ProcessGroup | None = None, *,
                      causal: bool = True, window: int | None = None) -> Tensor:
    """q, k, v: (B, T_local, H, d) with H % P == 0; ``q_pos`` the local rows' global positions
    (the same for K / V).  Returns (B, T_local, H, d)."""
    ws = dist.get_world_size(group)
    if q.shape[2] % ws or k.shape[2] % ws:
        raise ValueError(f"heads ({q.shape[2]}, {k.shape[2]}) must be divisible by the group size {ws}")
    pos = torch.empty(ws * q_pos.numel(), dtype=q_pos.dtype, device=q_pos.device)
    _gather_pos(pos, q_pos, group)
    qh, kh, vh = (_SeqToHead.apply(t, group) for t in (q, k, v))
    out = local_attention(qh, kh, vh, pos, pos, causal=causal, window=window)
    return _HeadToSeq.apply(out, group)


def _gather_pos(out: Tensor, pos: Tensor, group: dist.ProcessGroup | None) -> None:
    parts = [torch.empty_like(pos) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, pos.contiguous(), group=group)
    out.copy_(torch.cat(parts))


class _RingHop(torch.autograd.Function):
    """Send x to rank + 1, receive from rank - 1; the backward goes the other way."""

    @staticmethod
    def forward(ctx, x: Tensor, group):  # type: ignore[override]
        ctx.group = group
        return _hop(x, group, +1)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return _hop(g, ctx.group, -1), None


def _hop(x: Tensor, group: dist.ProcessGroup | None, direction: int) -> Tensor:
    rank, ws = dist.get_rank(group), dist.get_world_size(group)
    dst, src = (rank + direction) % ws, (rank - direction) % ws
    if group is not None:
        dst, src = dist.get_global_rank(group, dst), dist.get_global_rank(group, src)
    x = x.contiguous()
    out = torch.empty_like(x)
    for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, x, dst, group),
                                       dist.P2POp(dist.irecv, out, src, group)]):
        req.wait()
    return out


def ring_attention(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, group: dist.ProcessGroup | None = None, *,
                   causal: bool = True, window: int | None = None) -> Tensor:
    """q, k, v: (B, T_local, H, d) local shards with global positions ``q_pos`` (also the
    positions of the local K / V).  Returns (B, T_local, H, d)."""
    ws = dist.get_world_size(group)
    scale = 1.0 / math.sqrt(q.shape[-1])
    # the K/V positions travel with the blocks (they are a tiny integer tensor)
    kv = torch.cat([k, v], dim=-1)
    k_pos = q_pos
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.full((q.shape[0], q.shape[2], q.shape[1]), float("-inf"), device=q.device)
    d = q.shape[-1]
    for step in range(ws):
        kb, vb = kv[..., :d], kv[..., d:]
        hidden = causal and bool((k_pos.min() > q_pos.max()).item())
        if window is not None:
            hidden = hidden or bool((k_pos.max() <= q_pos.min() - window).item())
        if hidden:
            # keep this block in the graph (zero weight) so every rank's ring hop takes part in
            # the backward: the hops exchange gradients point-to-point in lockstep
            out = out + 0.0 * kv.float().sum()
        else:
            o_b, l_b = _block(q, kb, vb, q_pos, k_pos, causal, window, scale)
            new = torch.logaddexp(lse, l_b)
            safe = torch.where(torch.isfinite(new), new, torch.zeros_like(new))
            w_old = torch.exp(lse - safe).transpose(1, 2)[..., None]
            w_new = torch.exp(l_b - safe).transpose(1, 2)[..., None]
            out = out * w_old + o_b * w_new
            lse = new
        if step + 1 < ws:
            kv = _RingHop.apply(kv, group)
            k_pos = _hop(k_pos, group, +1)
    return out.to(q.dtype)


def zigzag_positions(t_total: int, rank: int, ws: int, device: torch.device | None = None) -> Tensor:
    """Global positions of rank ``rank``'s rows under zigzag sharding: blocks ``rank`` and
    ``2 ws - 1 - rank`` of ``2 ws`` equal blocks."""
    if t_total % (2 * ws):
        raise ValueError("sequence length must be a multiple of 2 x group size")
    c = t_total // (2 * ws)
    a, b = rank * c, (2 * ws - 1 - rank) * c
    return torch.cat([torch.arange(a, a + c, device=device), torch.arange(b, b + c, device=device)])


def contiguous_positions(t_total: int, rank: int, ws: int, device: torch.device | None = None) -> Tensor:
    c = t_total // ws
    return torch.arange(rank * c, (rank + 1) * c, device=device)


__all__ = ["contiguous_positions", "local_attention", "ring_attention", "ulysses_attention", "zigzag_positions"]

"""Pipeline parallelism: the block stack split into contiguous stages, one per rank,
driven by a 1F1B schedule with point-to-point send/recv of the mHC residual stream
(absent in the reference, which plans DualPipe; the build plan keeps pipeline traffic
on NCCL p2p, overlapped with compute).

Stage ``s`` of ``S`` owns blocks ``[s*L/S, (s+1)*L/S)``; stage 0 also owns the input
embedding, the last stage the final norm, LM head, MTP heads and the loss.  Between
stages travels ``x`` of shape (micro-batch, T, n_hc, D) forward and its gradient
backward.  Every stage gets the micro-batch's token ids (the hash router and the MTP
targets need them; ids are tiny next to activations).

1F1B: stage ``s`` runs ``min(S-s-1, M)`` warm-up forwards, then alternates one
forward and one backward, then drains the remaining backwards; at most ``S - s``
micro-batches of activations are alive on stage s.  Sends are non-blocking
(``isend``), receives blocking; every stage issues its sends and receives in schedule
order, so matching pairs always meet.

With tied embeddings the first and last stages both hold the embedding matrix;
``sync_tied_embedding`` sums its gradient over the two after the schedule.

Context parallelism inside each stage (config 4's PP x CP layout): with ``cp_group`` every
stage's sequence is split over that group as in ``parallel.cp`` (each rank holds a
contiguous shard; attention exchanges the window halo and the compressed entries), the
stage boundary carries the shard's residual stream to the same CP rank of the next stage
(the pipeline group links the ranks with one CP index), and the last stage's loss is this
shard's share of the global mean (``cp_lm_share``).  ``sync_cp_grads`` then sums the
stage's gradients over the CP group.  Every CP rank of a stage runs the same schedule, so
their attention collectives pair up in order.
"""

from __future__ import annotations

import contextlib
from collections.abc import Callable

import torch
import torch.distributed as dist
from torch import Tensor, nn

from saint_llm_b200.models.mhc import MHC


def stage_bounds(n_layers: int, n_stages: int, stage: int) -> tuple[int, int]:
    base, extra = divmod(n_layers, n_stages)
    start = stage * base + min(stage, extra)
    return start, start + base + (1 if stage < extra else 0)


class PipelineStage:
    def __init__(self, model: nn.Module, group: dist.ProcessGroup | None = None, *, prune: bool = False,
                 cp_group: dist.ProcessGroup | None = None) -> None:
        self.model, self.group = model, group
        self.cp_group = cp_group
        self.stage = dist.get_rank(group)
        self.n_stages = dist.get_world_size(group)
        self.first, self.last = self.stage == 0, self.stage == self.n_stages - 1
        self.lo, self.hi = stage_bounds(len(model.blocks), self.n_stages, self.stage)  # type: ignore[arg-type]
        if prune:
            for i in range(len(model.blocks)):  # type: ignore[arg-type]
                if not self.lo <= i < self.hi:
                    model.blocks[i] = nn.Identity()  # type: ignore[index]

    def _peer(self, s: int) -> int:
        return dist.get_global_rank(self.group, s) if self.group is not None else s

    def local_ids(self, ids: Tensor) -> Tensor:
        """The tokens this rank computes: its CP shard of ``ids`` (all of them without CP)."""
        if self.cp_group is None:
            return ids
        from saint_llm_b200.parallel.cp import cp_shard

        return cp_shard(ids, self.cp_group)

    def forward(self, ids: Tensor, x_in: Tensor | None) -> Tensor:
        """``ids``: the micro-batch's full (B, T) token ids."""
        m = self.model
        local = self.local_ids(ids)
        if self.first:
            x = MHC.expand(m._embed_inputs(local, None, None), m.cfg.mhc.expansion_factor)  # type: ignore[attr-defined]
        else:
            assert x_in is not None
            x = x_in
        vis = local == m.cfg.tokenizer_slots.image_pad  # type: ignore[attr-defined]
        bundle = None
        if self.cp_group is not None:
            from saint_llm_b200.parallel.cp import CPBundle

            bundle = CPBundle(m, self.cp_group, local.shape[1])
        from saint_llm_b200.parallel.cp import balance_over

        with balance_over(m, self.cp_group) if self.cp_group is not None else contextlib.nullcontext():
            for i in range(self.lo, self.hi):
                view = bundle.for_layer(i) if bundle is not None else None
                x = m.blocks[i](x, token_ids=local, is_visual=vis, kv_cache_layer=view)  # type: ignore[index]
        return x

    def loss(self, ids: Tensor, x: Tensor, loss_fn: Callable[[nn.Module, Tensor, Tensor], Tensor]) -> Tensor:
        """Last stage: ``loss_fn(model, final-normed hidden, ids)``."""
        h = self.model.final_norm(MHC.collapse(x))  # type: ignore[attr-defined]
        return loss_fn(self.model, h, ids)


def aux_losses(model: nn.Module, lo: int, hi: int) -> Tensor | None:
    total = None
    for i in range(lo, hi):
        a = getattr(model.blocks[i].moe, "_last_aux_loss", None)  # type: ignore[index]
        if isinstance(a, Tensor) and a.requires_grad:
            total = a if total is None else total + a
    return total


def default_lm_loss(model: nn.Module, h: Tensor, ids: Tensor) -> Tensor:
    """Main next-token CE (mean over the micro-batch's positions)."""
    logits = model.logits(h[:, :-1]).float()  # type: ignore[attr-defined]
    return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))


def cp_lm_share(group: dist.ProcessGroup | None) -> Callable[[nn.Module, Tensor, Tensor], Tensor]:
    """The main next-token CE for a CP-sharded last stage: ``h`` holds this rank's shard of the
    positions, ``ids`` the full sequence (the shard's last target is the next shard's first
    token); returns this shard's share of the global mean (the sum over the group is the loss)."""

    def loss(model: nn.Module, h: Tensor, ids: Tensor) -> Tensor:
        from saint_llm_b200.parallel.cp import shard_loss

        return shard_loss(model, h, ids, dist.get_rank(group) * h.shape[1])

    return loss


@torch.no_grad()
def sync_cp_grads(stage: PipelineStage) -> None:
    """Sum the stage's parameter gradients over its CP group (each rank's are the share of
    its own tokens).  A parameter can have a gradient on one shard and none on another (an
    expert no token of that shard was routed to), so the ranks first agree on which
    parameters take part; those nobody touched keep no gradient (the optimizer skips them)."""
    if stage.cp_group is None:
        return
    params = [p for p in stage.model.parameters() if p.requires_grad]
    if not params:
        return
    dev = params[0].device
    used = torch.tensor([p.grad is not None for p in params], dtype=torch.int32, device=dev)
    dist.all_reduce(used, group=stage.cp_group)
    grads = []
    for p, u in zip(params, used.tolist(), strict=True):
        if u:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            grads.append(p.grad)
    if grads:
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        dist.all_reduce(flat, group=stage.cp_group)
        off = 0
        for g in grads:
            g.copy_(flat[off:off + g.numel()].view_as(g))
            off += g.numel()


def run_1f1b(stage: PipelineStage, micro_ids: list[Tensor], *,
             loss_fn: Callable[[nn.Module, Tensor, Tensor], Tensor] | None = None,
             aux_weight: float = 0.0) -> Tensor | None:
    """One pipelined forward+backward over ``micro_ids``; gradients accumulate in the
    stage's parameters (each micro-batch's loss is divided by M).  Returns the mean loss
    on the last stage (with CP: this rank's share of it), None elsewhere.  ``loss_fn``
    defaults to ``default_lm_loss`` (``cp_lm_share`` with a CP group)."""
    if loss_fn is None:
        loss_fn = default_lm_loss if stage.cp_group is None else cp_lm_share(stage.cp_group)
    m = stage.model
    M = len(micro_ids)
    cfg = m.cfg  # type: ignore[attr-defined]
    dtype = next(m.parameters()).dtype
    dev = micro_ids[0].device
    n_warm = min(stage.n_stages - stage.stage - 1, M)
    saved: dict[int, tuple[Tensor | None, Tensor]] = {}
    pending: list = []
    losses: list[Tensor] = []

    def shape(ids: Tensor) -> tuple[int, ...]:
        local = stage.local_ids(ids)
        return (local.shape[0], local.shape[1], cfg.mhc.expansion_factor, cfg.hidden_dim)

    def fwd(i: int) -> None:
        ids = micro_ids[i]
        x_in = None
        if not stage.first:
            x_in = torch.empty(shape(ids), dtype=dtype, device=dev)
            dist.recv(x_in, stage._peer(stage.stage - 1), group=stage.group)
            x_in.requires_grad_(True)
        out = stage.forward(ids, x_in)
        aux = aux_losses(m, stage.lo, stage.hi)
        if stage.last:
            loss = stage.loss(ids, out, loss_fn)
            losses.append(loss.detach())
            out = loss / M
        if aux is not None and aux_weight:
            out = (out, aux * (aux_weight / M))  # type: ignore[assignment]
        saved[i] = (x_in, out)  # type: ignore[assignment]
        if not stage.last:
            y = out[0] if isinstance(out, tuple) else out
            pending.append(dist.isend(y.detach().contiguous(), stage._peer(stage.stage + 1), group=stage.group))

    def bwd(i: int) -> None:
        x_in, out = saved.pop(i)
        outs, grads = [], []
        y, aux = (out if isinstance(out, tuple) else (out, None))
        if stage.last:
            outs.append(y)
            grads.append(None)
        else:
            g = torch.empty_like(y)
            dist.recv(g, stage._peer(stage.stage + 1), group=stage.group)
            outs.append(y)
            grads.append(g)
        if aux is not None:
            outs.append(aux)
            grads.append(None)
        torch.autograd.backward(outs, grads)
        if not stage.first:
            assert x_in is not None
            pending.append(dist.isend(x_in.grad.contiguous(), stage._peer(stage.stage - 1), group=stage.group))

    for i in range(n_warm):
        fwd(i)
    for i in range(M - n_warm):
        fwd(n_warm + i)
        bwd(i)
    for i in range(M - n_warm, M):
        bwd(i)
    for req in pending:
        req.wait()
    return torch.stack(losses).mean() if losses else None


def sync_tied_embedding(stage: PipelineStage) -> None:
    """Sum the tied embedding / LM-head gradient over the first and last stages (a P2P
    exchange between the two; the middle stages do nothing)."""
    m = stage.model
    if stage.n_stages == 1 or not (stage.first or stage.last) or not m.cfg.tie_word_embeddings:  # type: ignore[attr-defined]
        return
    w = m.embed.weight  # type: ignore[attr-defined]
    g = getattr(w, "main_grad", None)
    if g is None:
        if w.grad is None:
            w.grad = torch.zeros_like(w)
        g = w.grad
    peer = stage._peer(stage.n_stages - 1 if stage.first else 0)
    mine = g.detach().float().contiguous().clone()
    other = torch.empty_like(mine)
    for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, mine, peer, stage.group),
                                     dist.P2POp(dist.irecv, other, peer, stage.group)]):
        r.wait()
    g.copy_(mine + other)


__all__ = ["PipelineStage", "aux_losses", "cp_lm_share", "default_lm_loss", "run_1f1b", "stage_bounds", "sync_cp_grads",
           "sync_tied_embedding"]

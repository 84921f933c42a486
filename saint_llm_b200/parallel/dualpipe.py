"""DualPipe-V: a V-shaped pipeline schedule (absent in the reference, which lists
DualPipe / DualPipeV as planned in ``distributed/__init__.py:9-13``).  Pipeline traffic is
NCCL (or gloo) point-to-point, posted at the end of each tick and waited for only by the
op that consumes the tensor, so a tick's exchange overlaps the following ticks' compute.

Placement.  The block stack is cut into ``2P`` virtual stages for ``P`` ranks; rank ``r``
holds virtual stage ``r`` (chunk 0) and virtual stage ``2P-1-r`` (chunk 1).  A micro-batch
runs down the ranks through chunk 0 and back up through chunk 1, so:

* rank 0 holds both ends -- the input embedding, the final norm, LM head, MTP heads and the
  loss -- and a tied embedding needs no gradient exchange;
* rank ``P-1`` hands chunk 0's output to its own chunk 1 without communication;
* every rank holds two chunks, so a rank that would idle in a one-directional pipeline
  (waiting for the first backward) works on the other chunk instead.

Schedule.  Every rank computes the same timetable by simulating the pipeline in ticks: in
each tick a rank runs at most one op, ``F(v, i)`` or ``B(v, i)`` (forward / backward of
virtual stage ``v`` for micro-batch ``i``), whose inputs were produced in an earlier tick.
Ready backwards go first (oldest micro-batch first), then forwards, preferring chunk 1 so
finished activations leave the pipeline early; a new micro-batch enters rank ``r`` only
while fewer than ``2P - r`` micro-batches are between its chunk-0 forward and backward,
which bounds the activations alive on a rank.  After each tick the activations and input
gradients that cross ranks are posted in one grouped ``batch_isend_irecv``: every rank posts
its sends and receives of that tick in one canonical order, so matching pairs always meet.
Nothing waits at the end of the tick: a receive is waited for by the op that consumes it
(always in a later tick), and the sends are waited for after the last tick (their tensors
are kept alive until then).  No deadlock: posting never blocks, and an op at tick t waits only
for a message its peer posted at the end of a tick before t, which the peer reaches after
waits of the same kind for even earlier ticks.

Gradients accumulate in the parameters as with ``run_1f1b`` (each micro-batch's loss is
divided by ``M``); the result equals the non-pipelined step.

Context parallelism inside the chunks (``cp_group``) works as in ``parallel.pipeline``: each
chunk's sequence is this rank's CP shard, the loss on rank 0 is the shard's share
(``cp_lm_share``), and ``pipeline.sync_cp_grads(pipe)`` sums the gradients over the CP group
afterwards.  The CP ranks of one pipeline rank follow the same timetable, so their attention
collectives pair up.
"""

from __future__ import annotations

import contextlib
from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor, nn

from saint_llm_b200.models.mhc import MHC
from saint_llm_b200.parallel.pipeline import aux_losses, cp_lm_share, default_lm_loss, stage_bounds


@dataclass(frozen=True)
class Op:
    kind: str  # "F" or "B"
    v: int     # virtual stage
    i: int     # micro-batch


def owner(v: int, n_ranks: int) -> int:
    """Rank holding virtual stage ``v`` of ``2 * n_ranks``."""
    return v if v < n_ranks else 2 * n_ranks - 1 - v


def build_schedule(n_ranks: int, n_micro: int) -> list[list[Op | None]]:
    """Per tick, the op each rank runs (None = idle); identical on every rank."""
    P, M, S = n_ranks, n_micro, 2 * n_ranks
    f_done: set[tuple[int, int]] = set()
    b_done: set[tuple[int, int]] = set()
    cap = [2 * P - r for r in range(P)]
    ticks: list[list[Op | None]] = []
    while len(b_done) < S * M:
        row: list[Op | None] = []
        for r in range(P):
            chunks = (r, S - 1 - r)
            op = None
            for i in range(M):  # ready backwards, oldest first
                for v in chunks:
                    if (v, i) in f_done and (v, i) not in b_done and (v == S - 1 or (v + 1, i) in b_done):
                        op = Op("B", v, i)
                        break
                if op:
                    break
            if op is None:
                inflight = sum(1 for i in range(M) if (r, i) in f_done and (r, i) not in b_done)
                for i in range(M):
                    for v in (chunks[1], chunks[0]):
                        if (v, i) in f_done or not (v == 0 or (v - 1, i) in f_done):
                            continue
                        if v == r and inflight >= cap[r]:
                            continue
                        op = Op("F", v, i)
                        break
                    if op:
                        break
            row.append(op)
        if all(o is None for o in row):
            raise RuntimeError("pipeline schedule stalled")  # cannot happen: the oldest micro-batch can always move
        for op in row:
            if op is not None:
                (f_done if op.kind == "F" else b_done).add((op.v, op.i))
        ticks.append(row)
    return ticks


def messages(row: list[Op | None], n_ranks: int) -> list[tuple[int, int, str, int]]:
    """(src, dst, kind, micro-batch) of the tensors this tick's ops send to another rank:
    a forward sends its output to the next virtual stage, a backward its input gradient
    to the previous one.  Sorted canonically."""
    S = 2 * n_ranks
    out = []
    for op in row:
        if op is None:
            continue
        if op.kind == "F" and op.v + 1 < S:
            src, dst = owner(op.v, n_ranks), owner(op.v + 1, n_ranks)
            if src != dst:
                out.append((src, dst, "act", op.i))
        elif op.kind == "B" and op.v > 0:
            src, dst = owner(op.v, n_ranks), owner(op.v - 1, n_ranks)
            if src != dst:
                out.append((src, dst, "grad", op.i))
    return sorted(out)


class DualPipeV:
    """One rank's two chunks of ``model`` (``prune=True`` drops the other ranks' blocks)."""

    def __init__(self, model: nn.Module, group: dist.ProcessGroup | None = None, *, prune: bool = False,
                 cp_group: dist.ProcessGroup | None = None) -> None:
        self.model, self.group = model, group
        self.cp_group = cp_group
        self.rank = dist.get_rank(group)
        self.P = dist.get_world_size(group)
        n_layers = len(model.blocks)  # type: ignore[arg-type]
        self.bounds = {v: stage_bounds(n_layers, 2 * self.P, v) for v in (self.rank, 2 * self.P - 1 - self.rank)}
        if prune:
            keep = {i for lo, hi in self.bounds.values() for i in range(lo, hi)}
            for i in range(n_layers):
                if i not in keep:
                    model.blocks[i] = nn.Identity()  # type: ignore[index]

    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def local_ids(self, ids: Tensor) -> Tensor:
        if self.cp_group is None:
            return ids
        from saint_llm_b200.parallel.cp import cp_shard

        return cp_shard(ids, self.cp_group)

    def _forward(self, v: int, ids: Tensor, x: Tensor | None) -> Tensor:
        m = self.model
        local = self.local_ids(ids)
        if v == 0:
            x = MHC.expand(m._embed_inputs(local, None, None), m.cfg.mhc.expansion_factor)  # type: ignore[attr-defined]
        vis = local == m.cfg.tokenizer_slots.image_pad  # type: ignore[attr-defined]
        bundle = None
        if self.cp_group is not None:
            from saint_llm_b200.parallel.cp import CPBundle

            bundle = CPBundle(m, self.cp_group, local.shape[1])
        lo, hi = self.bounds[v]
        from saint_llm_b200.parallel.cp import balance_over

        with balance_over(m, self.cp_group) if self.cp_group is not None else contextlib.nullcontext():
            for j in range(lo, hi):
                view = bundle.for_layer(j) if bundle is not None else None
                x = m.blocks[j](x, token_ids=local, is_visual=vis, kv_cache_layer=view)  # type: ignore[index]
        assert x is not None
        return x


def run_dualpipe(pipe: DualPipeV, micro_ids: list[Tensor], *,
                 loss_fn: Callable[[nn.Module, Tensor, Tensor], Tensor] | None = None,
                 aux_weight: float = 0.0) -> Tensor | None:
    """One DualPipe-V forward+backward over ``micro_ids``; returns the mean loss on rank 0
    (with CP: this rank's share of it).  ``loss_fn`` defaults to ``default_lm_loss``
    (``cp_lm_share`` with a CP group)."""
    if loss_fn is None:
        loss_fn = default_lm_loss if pipe.cp_group is None else cp_lm_share(pipe.cp_group)
    m = pipe.model
    P, S, M, rank = pipe.P, 2 * pipe.P, len(micro_ids), pipe.rank
    cfg = m.cfg  # type: ignore[attr-defined]
    dtype = next(m.parameters()).dtype
    dev = micro_ids[0].device
    ticks = build_schedule(P, M)
    inbox: dict[tuple[str, int, int], Tensor] = {}   # (kind, virtual stage that consumes it, i)
    arriving: dict[tuple[str, int, int], list] = {}  # pending receive(s) of an inbox entry
    in_flight: list[tuple[list, Tensor]] = []         # posted sends and the tensors they read

    # a work is waited for once (gloo's p2p waits are not idempotent); the dict keeps every
    # waited work alive, so no later work can reuse its id
    waited: dict[int, object] = {}

    def wait(w: object) -> None:
        if id(w) not in waited:
            waited[id(w)] = w
            w.wait()  # type: ignore[attr-defined]

    def take(key: tuple[str, int, int]) -> Tensor:
        for w in arriving.pop(key, []):
            wait(w)
        return inbox.pop(key)

    saved: dict[tuple[int, int], tuple[Tensor | None, Tensor | tuple[Tensor, Tensor]]] = {}
    losses: list[Tensor] = []
    dist.barrier(group=pipe.group)  # every rank's communicator exists before the first grouped p2p

    def shape(i: int) -> tuple[int, ...]:
        ids = pipe.local_ids(micro_ids[i])
        return (ids.shape[0], ids.shape[1], cfg.mhc.expansion_factor, cfg.hidden_dim)

    for row in ticks:
        op = row[rank]
        produced: dict[tuple[str, int], Tensor] = {}
        if op is not None and op.kind == "F":
            ids = micro_ids[op.i]
            x_in = None
            if op.v > 0:
                x_in = take(("act", op.v, op.i)).detach().requires_grad_(True)
            out = pipe._forward(op.v, ids, x_in)
            aux = aux_losses(m, *pipe.bounds[op.v])
            if op.v == S - 1:
                h = m.final_norm(MHC.collapse(out))  # type: ignore[attr-defined]
                loss = loss_fn(m, h, ids)
                losses.append(loss.detach())
                out = loss / M
            saved[(op.v, op.i)] = (x_in, (out, aux * (aux_weight / M)) if aux is not None and aux_weight else out)
            if op.v + 1 < S:
                if owner(op.v + 1, P) == rank:
                    inbox[("act", op.v + 1, op.i)] = out.detach()
                else:
                    produced[("act", op.i)] = out.detach().contiguous()
        elif op is not None:
            x_in, out = saved.pop((op.v, op.i))
            y, aux = out if isinstance(out, tuple) else (out, None)
            outs, grads = [y], [None if op.v == S - 1 else take(("grad", op.v, op.i))]
            if aux is not None:
                outs.append(aux)
                grads.append(None)
            torch.autograd.backward(outs, grads)
            if op.v > 0:
                assert x_in is not None and x_in.grad is not None
                if owner(op.v - 1, P) == rank:
                    inbox[("grad", op.v - 1, op.i)] = x_in.grad
                else:
                    produced[("grad", op.i)] = x_in.grad.contiguous()
        # grouped exchange of this tick's cross-rank tensors, posted now, waited for by consumers
        p2p, keys = [], []
        for src, dst, kind, i in messages(row, P):
            if src == rank:
                p2p.append(dist.P2POp(dist.isend, produced[(kind, i)], pipe._peer(dst), pipe.group))
                keys.append(("send", produced[(kind, i)]))
            elif dst == rank:
                buf = torch.empty(shape(i), dtype=dtype, device=dev)
                # the consumer: the next virtual stage of a forward, the previous of a backward
                src_op = next(o for o in row if o is not None and owner(o.v, P) == src and o.i == i
                              and o.kind == ("F" if kind == "act" else "B"))
                v_dst = src_op.v + 1 if kind == "act" else src_op.v - 1
                inbox[(kind, v_dst, i)] = buf
                p2p.append(dist.P2POp(dist.irecv, buf, pipe._peer(src), pipe.group))
                keys.append(("recv", (kind, v_dst, i)))
        if p2p:
            reqs = dist.batch_isend_irecv(p2p)
            # gloo returns one work per op; NCCL coalesces the group into fewer works, each of
            # which then stands for every op of the tick
            per_op = len(reqs) == len(p2p)
            for j, (what, ref) in enumerate(keys):
                ws = [reqs[j]] if per_op else list(reqs)
                if what == "recv":
                    arriving[ref] = ws  # type: ignore[index]
                else:
                    in_flight.append((ws, ref))  # type: ignore[arg-type]
    for ws, _ in in_flight:
        for w in ws:
            wait(w)
    for ws in arriving.values():  # every receive has a consumer, so none is left; kept for safety
        for w in ws:
            wait(w)
    return torch.stack(losses).mean() if losses else None


__all__ = ["DualPipeV", "Op", "build_schedule", "messages", "owner", "run_dualpipe"]

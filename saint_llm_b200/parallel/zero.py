"""Hybrid ZeRO (Muon-aware): whole-tensor ownership of optimizer work per rank.

Planner (reference: ``saint_llm_distributed/zero.py:47-216``): Muon and AdamW parameters
are packed separately with greedy longest-processing-time bin packing (each item to the
currently lightest rank; Graham's 4/3 bound) on Muon cost ``n*m`` and AdamW cost ``numel``,
then merged per rank.

Runtime (``ZeroOptimizerSync``): the reference stops at the plan; here each replicated
parameter is owned by one rank.  After backward, gradients are *reduced* to their owners in
flat per-owner buckets (NCCL ``reduce``, summed then divided by the world size), only the
owner runs Muon/AdamW on a parameter (Newton-Schulz needs the whole matrix, so ownership is
per tensor), and the owner broadcasts the updated weights in the same buckets.  Traffic per
step equals one all-reduce (reduce + broadcast) while the optimizer work and the optimizer
state are split across ranks.

Overlapped mode (``overlap_groups``): the parameters are also partitioned into groups that
finish their gradients together (one transformer block each, plus a tail of everything
else).  During the last micro-batch of a step the caller marks ``final_micro``; a group's
reductions are issued from the block's backward hook the moment its gradients are written,
so they run on NCCL's stream while the backward of the earlier blocks continues.  Groups are
visited in backward order, which is the same on every rank, so every rank issues the same
collectives in the same order.
"""

from __future__ import annotations

import heapq
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

import torch
import torch.distributed as dist
from torch import Tensor


@dataclass(frozen=True)
class BucketAssignment:
    buckets: tuple[tuple[int, ...], ...]
    per_rank_cost: tuple[float, ...]

    @property
    def n_ranks(self) -> int:
        return len(self.buckets)

    @property
    def imbalance(self) -> float:
        if not self.per_rank_cost or max(self.per_rank_cost) <= 0:
            return 0.0
        hi = max(self.per_rank_cost)
        return (hi - min(self.per_rank_cost)) / hi

    def owner_of(self) -> dict[int, int]:
        return {i: r for r, b in enumerate(self.buckets) for i in b}


def pack_buckets_by_cost(costs: Sequence[float], n_buckets: int) -> BucketAssignment:
    if n_buckets <= 0:
        raise ValueError(f"n_buckets must be positive; got {n_buckets}")
    if any(c < 0 for c in costs):
        raise ValueError("costs must be non-negative")
    heap = [(0.0, r) for r in range(n_buckets)]
    members: list[list[int]] = [[] for _ in range(n_buckets)]
    load = [0.0] * n_buckets
    for i in sorted(range(len(costs)), key=lambda j: -float(costs[j])):
        c, r = heapq.heappop(heap)
        members[r].append(i)
        load[r] = c + float(costs[i])
        heapq.heappush(heap, (load[r], r))
    return BucketAssignment(tuple(tuple(sorted(m)) for m in members), tuple(load))


def muon_param_cost(t: Tensor) -> float:
    """Newton-Schulz cost proxy: n*m for a matrix (numel otherwise)."""
    return float(t.shape[0] * t.shape[1]) if t.dim() == 2 else float(t.numel())


def adamw_param_cost(t: Tensor) -> float:
    return float(t.numel())


def hybrid_zero_assign(params: Sequence[Tensor], optimizer_kinds: Sequence[Literal["muon", "adamw"]],
                       n_buckets: int) -> BucketAssignment:
    if len(params) != len(optimizer_kinds):
        raise ValueError(f"params length {len(params)} != optimizer_kinds length {len(optimizer_kinds)}")
    if n_buckets <= 0:
        raise ValueError(f"n_buckets must be positive; got {n_buckets}")
    bad = [i for i, k in enumerate(optimizer_kinds) if k not in ("muon", "adamw")]
    if bad:
        raise ValueError(f"optimizer_kinds entries must be 'muon' or 'adamw'; bad indices {bad}")
    pools = {k: [i for i, kk in enumerate(optimizer_kinds) if kk == k] for k in ("muon", "adamw")}
    cost = {"muon": muon_param_cost, "adamw": adamw_param_cost}
    buckets: list[list[int]] = [[] for _ in range(n_buckets)]
    load = [0.0] * n_buckets
    for kind, idx in pools.items():
        a = pack_buckets_by_cost([cost[kind](params[i]) for i in idx], n_buckets)
        for r in range(n_buckets):
            buckets[r] += [idx[j] for j in a.buckets[r]]
            load[r] += a.per_rank_cost[r]
    return BucketAssignment(tuple(tuple(sorted(b)) for b in buckets), tuple(load))


def _grad_buf(p: Tensor) -> Tensor:
    g = getattr(p, "main_grad", None)
    if g is None:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        g = p.grad
    return g


class ZeroOptimizerSync:
    """Owner-partitioned gradient reduction and weight broadcast for replicated parameters.

    ``params``: the replicated (data-parallel) parameters; ``kinds``: "muon"/"adamw" per
    parameter.  Use: backward -> ``reduce_grads()`` -> ``optimizer.step()`` (non-owned
    parameters have their gradient buffers zeroed and are skipped via ``owned``) ->
    ``broadcast_params()``.
    """

    def __init__(self, params: Sequence[Tensor], kinds: Sequence[Literal["muon", "adamw"]], *,
                 group: dist.ProcessGroup | None = None, bucket_bytes: int = 256 << 20,
                 world: int | None = None, rank: int | None = None) -> None:
        # world / rank override the process group's (ranks emulated in one process)
        self.group = group
        self.world = world if world is not None else (dist.get_world_size(group) if dist.is_initialized() else 1)
        self.rank = rank if rank is not None else (dist.get_rank(group) if dist.is_initialized() else 0)
        self.params = list(params)
        self.plan = hybrid_zero_assign(self.params, kinds, self.world)
        owner = self.plan.owner_of()
        self.owner = [owner[i] for i in range(len(self.params))]
        self.owned = {id(p) for i, p in enumerate(self.params) if self.owner[i] == self.rank}
        self._buckets: list[tuple[int, list[int]]] = []
        for r in range(self.world):
            cur: list[int] = []
            size = 0
            for i in self.plan.buckets[r]:
                cur.append(i)
                size += self.params[i].numel() * 4
                if size >= bucket_bytes:
                    self._buckets.append((r, cur))
                    cur, size = [], 0
            if cur:
                self._buckets.append((r, cur))

    # ------------------------------------------------------------ overlapped reduce
    def overlap_groups(self, groups: list[list[Tensor]]) -> None:
        """Partition the parameters into ``groups`` (each reduced from a backward hook) and
        a tail (the parameters in no group, reduced after the backward)."""
        index = {id(p): i for i, p in enumerate(self.params)}
        self._groups: list[list[tuple[int, list[int]]]] = []
        grouped: set[int] = set()
        for g in groups:
            idx = [index[id(p)] for p in g if id(p) in index]
            grouped.update(idx)
            self._groups.append(self._by_owner(idx))
        self._tail = self._by_owner([i for i in range(len(self.params)) if i not in grouped])
        self._done: set[int] = set()
        self.final_micro = False

    def _by_owner(self, idx: list[int]) -> list[tuple[int, list[int]]]:
        per: dict[int, list[int]] = {}
        for i in idx:
            per.setdefault(self.owner[i], []).append(i)
        return sorted(per.items())

    def group_done(self, g: int) -> None:
        """Backward hook of group ``g``: reduce its gradients now if this is the step's
        last micro-batch (each group once per step)."""
        if not self.final_micro or g in self._done or self.world == 1:
            return
        self._done.add(g)
        for owner, idx in self._groups[g]:
            self._reduce_bucket(owner, idx)

    def _reduce_bucket(self, owner: int, idx: list[int]) -> None:
        grads = [_grad_buf(self.params[i]) for i in idx]
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        dist.reduce(flat, dst=self._global_rank(owner), op=dist.ReduceOp.SUM, group=self.group)
        if owner == self.rank:
            flat.div_(self.world)
            off = 0
            for g in grads:
                g.copy_(flat[off:off + g.numel()].view_as(g))
                off += g.numel()
        else:
            for g in grads:
                g.zero_()

    @torch.no_grad()
    def finish_reduce(self) -> None:
        """After the backward of an overlapped step: reduce every group whose hook did not
        fire (in group order) and the tail, then re-arm for the next step."""
        if self.world > 1:
            for g in range(len(self._groups)):
                if g not in self._done:
                    for owner, idx in self._groups[g]:
                        self._reduce_bucket(owner, idx)
            for owner, idx in self._tail:
                self._reduce_bucket(owner, idx)
        self._done = set()
        self.final_micro = False

    def _global_rank(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    @torch.no_grad()
    def reduce_grads(self) -> None:
        """Sum each bucket's gradients onto its owner (mean over ranks); zero them elsewhere."""
        if self.world == 1:
            return
        for owner, idx in self._buckets:
            self._reduce_bucket(owner, idx)

    @torch.no_grad()
    def broadcast_params(self) -> None:
        if self.world == 1:
            return
        for owner, idx in self._buckets:
            ps = [self.params[i] for i in idx]
            flat = torch.cat([p.data.reshape(-1) for p in ps])
            dist.broadcast(flat, src=self._global_rank(owner), group=self.group)
            if owner != self.rank:
                off = 0
                for p in ps:
                    p.data.copy_(flat[off:off + p.numel()].view_as(p))
                    off += p.numel()

    def is_owned(self, p: Tensor) -> bool:
        return id(p) in self.owned


__all__ = ["BucketAssignment", "ZeroOptimizerSync", "adamw_param_cost", "hybrid_zero_assign", "muon_param_cost",
           "pack_buckets_by_cost"]

"""Hybrid ZeRO over NVLink peer memory (``csrc/zero.cu``): the owner-partitioned gradient
reduction and weight broadcast of ``parallel.zero`` without NCCL.

The reference stops at the planner (``distributed/src/saint_llm_distributed/zero.py:47-216``);
``ZeroOptimizerSync`` runs it with NCCL ``reduce`` / ``broadcast``.  Here the replicated
parameters and their fp32 ``main_grad`` buffers are re-homed into two symmetric arenas (same
layout on every rank, mapped into every peer), and:

* a block's gradients, once final (its backward hook during the step's last micro-batch, or
  after the backward), are announced to every rank with one flag store per peer; each owner
  then PULLS the block's owned gradients from all ranks with peer loads and sums them in rank
  order (mean over ranks), on a side stream that overlaps the rest of the backward;
* after the optimizer, each rank announces its updated parameters, and every rank pulls the
  parameters it does not own from their owners.

Each parameter crosses NVLink once per non-owner per step in each direction, as with NCCL's
reduce + broadcast, but every transfer is a kernel of this framework that starts the moment
its flags are set.  The ordering argument (why no arena is overwritten while a peer reads it)
is in ``csrc/zero.cu``.  Eager steps only (the epoch lives on the host).
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Literal

import torch
import torch.distributed as dist
from torch import Tensor

from saint_llm_b200.ops import backend, gemm
from saint_llm_b200.parallel.ep_p2p import EmulatedHeap, SymmetricHeap
from saint_llm_b200.parallel.zero import ZeroOptimizerSync

GRAD_ALIGN = 32        # floats (128 bytes) between gradient slots
PARAM_ALIGN = 128      # bytes between parameter slots
GRAD_CHUNK = 1 << 18   # floats per reduce chunk
PARAM_CHUNK = 1 << 20  # bytes per parameter chunk
MAX_SLOTS = 128
PARAM_SLOT = MAX_SLOTS - 1


def _pad(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class PeerZeroSync(ZeroOptimizerSync):
    """``ZeroOptimizerSync`` with the peer-memory transport.  Construct it BEFORE the
    ``main_grad`` buffers are attached (it creates them, inside its arena) and before any
    optimizer state exists (the parameters move into the arena)."""

    def __init__(self, params: Sequence[Tensor], kinds: Sequence[Literal["muon", "adamw"]], *,
                 group: dist.ProcessGroup | None = None, device: torch.device | None = None,
                 heap: SymmetricHeap | EmulatedHeap | None = None, timeout_s: float = 30.0,
                 reduce_blocks: int = 48) -> None:
        dev = device if device is not None else params[0].device
        heap = heap if heap is not None else SymmetricHeap(group, dev)
        super().__init__(params, kinds, group=group, world=heap.ws, rank=heap.rank)
        self.heap = heap
        self.device = dev
        self.timeout_ns = int(timeout_s * 1e9)
        self.reduce_blocks = reduce_blocks
        self.err = gemm.error_word(dev)
        self.goff: list[int] = []
        self.poff: list[int] = []
        g_total = p_total = 0
        for p in self.params:
            self.goff.append(g_total)
            g_total += _pad(p.numel(), GRAD_ALIGN)
            self.poff.append(p_total)
            p_total += _pad(p.numel() * p.element_size(), PARAM_ALIGN)
        self.garena = self.heap.alloc(max(g_total, GRAD_ALIGN) * 4)
        self.parena = self.heap.alloc(max(p_total, PARAM_ALIGN))
        self.flags = self.heap.alloc(MAX_SLOTS * 8 * 4)
        gl = self.garena.local.view(torch.float32)
        with torch.no_grad():
            for i, p in enumerate(self.params):
                if getattr(p, "main_grad", None) is not None:
                    raise ValueError("PeerZeroSync must be built before the main_grad buffers are attached")
                n = p.numel()
                p.main_grad = gl[self.goff[i]:self.goff[i] + n].view(p.shape)  # type: ignore[attr-defined]
                nb = n * p.element_size()
                home = self.parena.local[self.poff[i]:self.poff[i] + nb].view(p.dtype).view(p.shape)
                home.copy_(p.data)
                p.data = home
        self.epoch = 1
        self.side = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self._owned_chunks_all = self._grad_chunks([i for i in range(len(self.params)) if self.owner[i] == self.rank])
        self._param_chunks = self._pchunks([i for i in range(len(self.params)) if self.owner[i] != self.rank])

    # ------------------------------------------------------------------ tables
    def _grad_chunks(self, idx: list[int]) -> Tensor:
        rows = []
        for i in idx:
            off, n = self.goff[i], _pad(self.params[i].numel(), 4)
            for s in range(0, n, GRAD_CHUNK):
                rows.append((off + s, min(GRAD_CHUNK, n - s)))
        return torch.tensor(rows or [(0, 0)], dtype=torch.int64, device=self.device)[: len(rows)].contiguous()

    def _pchunks(self, idx: list[int]) -> Tensor:
        rows = []
        for i in idx:
            off, nb = self.poff[i], _pad(self.params[i].numel() * self.params[i].element_size(), 16)
            for s in range(0, nb, PARAM_CHUNK):
                rows.append((off + s, min(PARAM_CHUNK, nb - s), self.owner[i]))
        return torch.tensor(rows or [(0, 0, 0)], dtype=torch.int64, device=self.device)[: len(rows)].contiguous()

    def overlap_groups(self, groups: list[list[Tensor]]) -> None:
        super().overlap_groups(groups)
        if len(self._groups) + 2 > MAX_SLOTS:
            raise ValueError(f"at most {MAX_SLOTS - 2} overlap groups")
        mine = lambda pairs: [i for owner, idx in pairs if owner == self.rank for i in idx]  # noqa: E731
        self._gchunks = [self._grad_chunks(mine(g)) for g in self._groups]
        self._tchunks = self._grad_chunks(mine(self._tail))

    # ------------------------------------------------------------------ kernels
    def _flags_local(self) -> Tensor:
        return self.flags.local.view(torch.int32)

    def _signal(self, slot: int) -> None:
        backend.ext().zero_signal(self.flags.ptrs, slot, self.rank, self.epoch)

    def _pull(self, chunks: Tensor, slot: int, blocks: int) -> None:
        if chunks.numel():
            backend.ext().zero_pull_reduce(chunks, self.garena.ptrs, self.rank, 1.0 / self.world,
                                           self._flags_local(), slot, self.epoch, self.timeout_ns, blocks, self.err)

    def _reduce_slot(self, slot: int, chunks: Tensor, *, side: bool) -> None:
        """Announce this rank's gradients of ``slot`` and pull the owned ones (on the side
        stream when ``side``, after the announcement in the current stream)."""
        self._signal(slot)
        if side and self.side is not None:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(ev)
                self._pull(chunks, slot, self.reduce_blocks)
        else:
            self._pull(chunks, slot, 4 * self.reduce_blocks)

    # --------------------------------------------------------------- interface
    def group_done(self, g: int) -> None:
        if not self.final_micro or g in self._done or self.world == 1:
            return
        self._done.add(g)
        self._reduce_slot(g, self._gchunks[g], side=True)

    @torch.no_grad()
    def finish_reduce(self) -> None:
        if self.world > 1:
            for g in range(len(self._groups)):
                if g not in self._done:
                    self._reduce_slot(g, self._gchunks[g], side=False)
            self._reduce_slot(len(self._groups), self._tchunks, side=False)
            if self.side is not None:
                torch.cuda.current_stream().wait_stream(self.side)
        self._done = set()
        self.final_micro = False

    @torch.no_grad()
    def reduce_grads(self) -> None:
        if self.world == 1:
            return
        self._reduce_slot(0, self._owned_chunks_all, side=False)

    @torch.no_grad()
    def broadcast_params(self) -> None:
        if self.world == 1:
            return
        self.publish_params()
        self.pull_params()

    def publish_params(self) -> None:
        """Announce that this rank's owned parameters of the current step are updated."""
        self._signal(PARAM_SLOT)

    def pull_params(self) -> None:
        """Copy every parameter this rank does not own from its owner (waits for the owners'
        announcements), then advance the step epoch."""
        if self._param_chunks.numel():
            backend.ext().zero_pull_params(self._param_chunks, self.parena.ptrs, self.rank, self._flags_local(),
                                           PARAM_SLOT, self.epoch, self.timeout_ns, 4 * self.reduce_blocks, self.err)
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF

    def check(self) -> None:
        gemm.check_errors(self.device)

    def close(self) -> None:
        self.heap.close()


__all__ = ["PeerZeroSync"]

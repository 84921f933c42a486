"""Tensor-parallel reductions over NVLink peer memory (``csrc/tp.cu``, ``gemm_peer_push``).

The reference has no tensor parallelism (its only multi-GPU training path is FSDP2,
``distributed/src/saint_llm_distributed/__init__.py:9-13``); this is the peer-memory transport
of ``parallel.tp``.  Forward, the row-parallel output projection of a head-sharded attention
block is ONE tcgen05 GEMM whose epilogue stores every output tile into each TP peer's receive
slot while the remaining tiles are multiplied, followed by a reduce kernel that sums the ranks'
partials in rank order (bit-identical on every rank).  Backward, the input gradient of the
block (a sum over several GEMMs, so no single producer) is pushed by a copy kernel and reduced
the same way.  Both use one symmetric receive buffer (two parities) and per-source arrival
counters; see ``csrc/tp.cu`` for the protocol.  No NCCL call is on this path.

Calls must be issued in the same order on every rank (as collectives are).  The expected
arrival counts live on the host, so this transport is for eager steps (not CUDA-graph replay).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from saint_llm_b200.ops import backend, gemm
from saint_llm_b200.ops.linear import _bf16, accumulate_weight_grad
from saint_llm_b200.parallel.ep_p2p import EmulatedHeap, SymmetricHeap


class PeerTPComm:
    """Receive buffer, counters and call bookkeeping of one TP group.

    ``max_elems``: the largest reduced tensor (elements); a larger one raises."""

    def __init__(self, heap: SymmetricHeap | EmulatedHeap, max_elems: int, *, timeout_s: float = 30.0) -> None:
        self.heap = heap
        self.rank, self.ws = heap.rank, heap.ws
        self.slot = (int(max_elems) + 127) // 128 * 128
        self.recv = heap.alloc(2 * self.ws * self.slot * 2)
        self.cnt = heap.alloc(self.ws * 4)
        self.expect = [0] * self.ws
        self.calls = 0
        self.timeout_ns = int(timeout_s * 1e9)
        self.err = gemm.error_word(heap.device)

    @classmethod
    def create(cls, group: dist.ProcessGroup | None, device: torch.device, max_elems: int,
               timeout_s: float = 30.0) -> PeerTPComm:
        return cls(SymmetricHeap(group, device), max_elems, timeout_s=timeout_s)

    # ---------------------------------------------------------------- addresses
    def _parity(self) -> int:
        return self.calls % 2

    def _slot_addr(self, peer: int, src: int, parity: int) -> int:
        return self.recv.ptrs[peer] + ((parity * self.ws + src) * self.slot) * 2

    def _peers(self) -> list[int]:
        return [p for p in range(self.ws) if p != self.rank]

    def _targets(self) -> tuple[list[int], list[int]]:
        par = self._parity()
        peers = self._peers()
        return ([self._slot_addr(p, self.rank, par) for p in peers],
                [self.cnt.ptrs[p] + 4 * self.rank for p in peers])

    def _check(self, n: int) -> None:
        if n > self.slot:
            raise ValueError(f"TP reduction of {n} elements exceeds the receive slot ({self.slot})")
        if n % 8:
            raise ValueError("TP peer reductions need numel % 8 == 0")

    # ------------------------------------------------------------------ stages
    def produce_gemm(self, x2: Tensor, w: Tensor) -> Tensor:
        """out = x2 w^T with every tile pushed to the peers (first half of a call)."""
        out = torch.empty(x2.shape[0], w.shape[0], dtype=torch.bfloat16, device=x2.device)
        self._check(out.numel())
        slots, cnts = self._targets()
        grid = backend.ext().gemm_peer_push(_bf16(x2).contiguous(), _bf16(w).contiguous(), out, slots, cnts,
                                            self.err)
        self._arrive(grid)
        return out

    def produce_copy(self, x: Tensor) -> Tensor:
        """Push ``x`` (bf16) to the peers; returns the contiguous bf16 tensor to reduce into."""
        xb = _bf16(x).contiguous()
        if xb.data_ptr() == x.data_ptr():
            xb = xb.clone()  # reduced in place: keep the caller's tensor
        self._check(xb.numel())
        slots, cnts = self._targets()
        grid = backend.ext().tp_push(xb, slots, cnts)
        self._arrive(grid)
        return xb

    def _arrive(self, grid: int) -> None:
        # every peer ran the same producer with the same grid
        self.expect = [(e + int(grid)) & 0xFFFFFFFF if s != self.rank else e for s, e in enumerate(self.expect)]

    def reduce(self, x: Tensor) -> Tensor:
        """Second half of a call: x (the produced tensor) += the peers' partials, in place."""
        par = self._parity()
        block = self.recv.local[par * self.ws * self.slot * 2:(par + 1) * self.ws * self.slot * 2]
        backend.ext().tp_reduce(x, block, self.slot, self.cnt.local[:4 * self.ws].view(torch.int32),
                                self.expect, self.rank, self.timeout_ns, self.err)
        self.calls += 1
        return x

    def allreduce(self, x: Tensor) -> Tensor:
        return self.reduce(self.produce_copy(x))

    def gemm_allreduce(self, x2: Tensor, w: Tensor) -> Tensor:
        return self.reduce(self.produce_gemm(x2, w))

    def check(self) -> None:
        """Raise if a wait timed out (reads the error word: one host sync)."""
        gemm.check_errors(self.heap.device)

    def close(self) -> None:
        self.heap.close()


class _PeerRowParallelFn(torch.autograd.Function):
    """y = sum over TP ranks of x_r W_r^T (forward: fused GEMM + peer push, then the reduce);
    backward is local: dx = dy W_r, dW_r = dy^T x_r."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, comm: PeerTPComm) -> Tensor:  # type: ignore[override]
        k = x.shape[-1]
        x2 = _bf16(x.reshape(-1, k))
        y = comm.gemm_allreduce(x2, weight)
        ctx.save_for_backward(x2, weight)
        ctx.in_dtype = x.dtype
        return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x2, weight = ctx.saved_tensors
        dy2 = _bf16(dy.reshape(-1, weight.shape[0]))
        dx = gemm.gemm_nt(dy2, _bf16(weight).t()).reshape(*dy.shape[:-1], weight.shape[1])
        if ctx.in_dtype != torch.bfloat16:
            dx = dx.to(ctx.in_dtype)
        dw = accumulate_weight_grad(weight, dy2, x2) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _PeerCopyToTPFn(torch.autograd.Function):
    """Identity forward; the input gradient is summed over the TP group by the peer kernels."""

    @staticmethod
    def forward(ctx, x: Tensor, comm: PeerTPComm) -> Tensor:  # type: ignore[override]
        ctx.comm = comm
        return x

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        out = ctx.comm.allreduce(g)
        return out.view(g.shape).to(g.dtype), None


def peer_row_parallel(x: Tensor, weight: Tensor, comm: PeerTPComm) -> Tensor:
    return _PeerRowParallelFn.apply(x, weight, comm)


def peer_copy_to_tp(x: Tensor, comm: PeerTPComm) -> Tensor:
    return _PeerCopyToTPFn.apply(x, comm)


class PeerRowParallelLinear(torch.nn.Module):
    """Drop-in for the sharded ``final_proj`` of a TP attention block: same Parameter, forward
    through ``peer_row_parallel`` (the block's output needs no further reduction)."""

    def __init__(self, weight: torch.nn.Parameter, comm: PeerTPComm) -> None:
        super().__init__()
        self.weight = weight
        self.in_features, self.out_features = weight.shape[1], weight.shape[0]
        self._comm = [comm]  # not a submodule

    def forward(self, x: Tensor) -> Tensor:
        return peer_row_parallel(x, self.weight, self._comm[0])


__all__ = ["PeerRowParallelLinear", "PeerTPComm", "peer_copy_to_tp", "peer_row_parallel"]

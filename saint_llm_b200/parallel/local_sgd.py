"""Communication-light outer loops: DiLoCo (SGD + Nesterov outer step) and NoLoCo (AdamW
outer step) over pseudo-gradients ``snapshot - current`` reduced across peers
(reference: ``saint_llm_distributed/diloco.py``, ``noloco.py``).

Reducers: identity (single node), ``AllReduceReducer`` (one flat NCCL/gloo all-reduce of all
pseudo-gradients -- the production path), and the in-process recursive-doubling ring used
as ground truth for gossip-style averaging (``ring_all_reduce``, ``RingAllReduceSimulator``).
"""

from __future__ import annotations

import math
import threading
from collections.abc import Iterable
from dataclasses import dataclass
from typing import Protocol

import torch
import torch.distributed as dist
from torch import Tensor


class PseudoGradientReducer(Protocol):
    def reduce(self, tensors: list[Tensor]) -> list[Tensor]: ...


class IdentityReducer:
    def reduce(self, tensors: list[Tensor]) -> list[Tensor]:
        return tensors


class AllReduceReducer:
    """Mean over the process group with a single flattened all-reduce."""

    def __init__(self, group: dist.ProcessGroup | None = None) -> None:
        self.group = group

    def reduce(self, tensors: list[Tensor]) -> list[Tensor]:
        if not tensors:
            return []
        flat = torch.cat([t.reshape(-1).float() for t in tensors])
        dist.all_reduce(flat, group=self.group)
        flat /= dist.get_world_size(self.group)
        out, off = [], 0
        for t in tensors:
            out.append(flat[off:off + t.numel()].view_as(t).to(t.dtype))
            off += t.numel()
        return out


def ring_log2_rounds(n_peers: int) -> int:
    return 0 if n_peers <= 1 else max(1, math.ceil(math.log2(n_peers)))


def ring_all_reduce(inputs_per_peer: list[list[Tensor]]) -> list[list[Tensor]]:
    """Recursive doubling: in round k peer i averages with peer i XOR 2^k (power-of-two N) or
    (i + 2^k) mod N otherwise.  Exact mean for power-of-two N."""
    n = len(inputs_per_peer)
    if n <= 1:
        return [list(p) for p in inputs_per_peer]
    state = [[t.detach().clone() for t in peer] for peer in inputs_per_peer]
    pow2 = n & (n - 1) == 0
    for k in range(ring_log2_rounds(n)):
        d = 1 << k
        partner = [(i ^ d) if pow2 else (i + d) % n for i in range(n)]
        state = [[(a + b) / 2 for a, b in zip(state[i], state[partner[i]], strict=True)] for i in range(n)]
    return state


class RingAllReduceSimulator:
    """Threads call ``peer_reducer(i).reduce(tensors)``; the last arrival computes the ring
    result and wakes everyone (a reusable barrier per round)."""

    def __init__(self, n_peers: int) -> None:
        if n_peers <= 0:
            raise ValueError(f"n_peers must be positive; got {n_peers}")
        self._n = n_peers
        self._cv = threading.Condition()
        self._inputs: list[list[Tensor] | None] = [None] * n_peers
        self._outputs: list[list[Tensor]] | None = None
        self._taken = 0
        self._generation = 0

    @property
    def n_peers(self) -> int:
        return self._n

    def peer_reducer(self, peer_index: int) -> PeerReducer:
        if not 0 <= peer_index < self._n:
            raise ValueError(f"peer_index {peer_index} out of range [0, {self._n})")
        return PeerReducer(self, peer_index)

    def _submit(self, i: int, tensors: list[Tensor]) -> list[Tensor]:
        with self._cv:
            while self._outputs is not None:  # previous round still being collected
                self._cv.wait()
            gen = self._generation
            self._inputs[i] = list(tensors)
            if all(x is not None for x in self._inputs):
                self._outputs = ring_all_reduce(self._inputs)  # type: ignore[arg-type]
                self._cv.notify_all()
            while self._outputs is None or self._generation != gen:
                self._cv.wait()
            out = self._outputs[i]
            self._taken += 1
            if self._taken == self._n:
                self._inputs, self._outputs, self._taken = [None] * self._n, None, 0
                self._generation += 1
                self._cv.notify_all()
            return out

    def run_round(self, inputs_per_peer: list[list[Tensor]]) -> list[list[Tensor]]:
        if len(inputs_per_peer) != self._n:
            raise ValueError(f"expected {self._n} peers; got {len(inputs_per_peer)}")
        return ring_all_reduce(inputs_per_peer)


class PeerReducer:
    def __init__(self, sim: RingAllReduceSimulator, index: int) -> None:
        self._sim, self._i = sim, index

    def reduce(self, tensors: list[Tensor]) -> list[Tensor]:
        return self._sim._submit(self._i, tensors)


class _OuterLoop:
    def __init__(self, params: Iterable[torch.nn.Parameter], inner_steps: int,
                 reducer: PseudoGradientReducer) -> None:
        self._params = list(params)
        self._reducer = reducer
        self._inner_steps = inner_steps
        self._snapshot = [p.detach().clone() for p in self._params]
        self._inner_count = 0

    def inner_step(self) -> None:
        self._inner_count += 1

    @property
    def should_sync(self) -> bool:
        return self._inner_count >= self._inner_steps

    def _pseudo_grads(self) -> list[Tensor]:
        return self._reducer.reduce([s - p.detach() for s, p in zip(self._snapshot, self._params, strict=True)])

    def _set(self, i: int, new: Tensor) -> None:
        self._params[i].data.copy_(new)
        self._snapshot[i] = new.detach().clone()


@dataclass
class DiLoCoConfig:
    inner_steps: int = 100
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    nesterov: bool = True


class DiLoCo(_OuterLoop):
    def __init__(self, params: Iterable[torch.nn.Parameter], cfg: DiLoCoConfig, *,
                 reducer: PseudoGradientReducer | None = None) -> None:
        super().__init__(params, cfg.inner_steps, reducer or IdentityReducer())
        self.cfg = cfg
        self._momentum = [torch.zeros_like(p) for p in self._params]

    @torch.no_grad()
    def outer_sync(self) -> None:
        c = self.cfg
        for i, g in enumerate(self._pseudo_grads()):
            buf = self._momentum[i].mul_(c.outer_momentum).add_(g)
            upd = g + c.outer_momentum * buf if c.nesterov else buf
            self._set(i, self._snapshot[i] - c.outer_lr * upd)
        self._inner_count = 0

    def state_dict(self) -> dict[str, object]:
        return {"snapshot": [s.clone() for s in self._snapshot], "momentum_buffer": [m.clone() for m in self._momentum],
                "inner_count": self._inner_count}

    def load_state_dict(self, state: dict[str, object]) -> None:
        if not isinstance(state.get("snapshot"), list) or not isinstance(state.get("momentum_buffer"), list):
            raise TypeError("DiLoCo state_dict has wrong shape")
        self._snapshot = list(state["snapshot"])  # type: ignore[arg-type]
        self._momentum = list(state["momentum_buffer"])  # type: ignore[arg-type]
        self._inner_count = int(state.get("inner_count", 0))  # type: ignore[arg-type]


@dataclass
class NoLoCoConfig:
    inner_steps: int = 500
    outer_lr: float = 1e-3
    outer_beta1: float = 0.9
    outer_beta2: float = 0.95
    outer_eps: float = 1e-8
    outer_weight_decay: float = 0.0


class NoLoCo(_OuterLoop):
    def __init__(self, params: Iterable[torch.nn.Parameter], cfg: NoLoCoConfig, *,
                 reducer: PseudoGradientReducer) -> None:
        super().__init__(params, cfg.inner_steps, reducer)
        self.cfg = cfg
        self._m = [torch.zeros_like(p) for p in self._params]
        self._v = [torch.zeros_like(p) for p in self._params]
        self._step = 0

    @torch.no_grad()
    def outer_sync(self) -> None:
        c = self.cfg
        grads = self._pseudo_grads()
        self._step += 1
        lr_t = c.outer_lr * math.sqrt(1 - c.outer_beta2 ** self._step) / (1 - c.outer_beta1 ** self._step)
        for i, g in enumerate(grads):
            self._m[i].mul_(c.outer_beta1).add_(g, alpha=1 - c.outer_beta1)
            self._v[i].mul_(c.outer_beta2).addcmul_(g, g, value=1 - c.outer_beta2)
            new = self._snapshot[i] - lr_t * self._m[i] / (self._v[i].sqrt() + c.outer_eps)
            if c.outer_weight_decay > 0:
                new = new * (1 - c.outer_lr * c.outer_weight_decay)
            self._set(i, new)
        self._inner_count = 0

    def state_dict(self) -> dict[str, object]:
        return {"snapshot": [s.clone() for s in self._snapshot], "m": [m.clone() for m in self._m],
                "v": [v.clone() for v in self._v], "inner_count": self._inner_count, "step": self._step}

    def load_state_dict(self, state: dict[str, object]) -> None:
        if not all(isinstance(state.get(k), list) for k in ("snapshot", "m", "v")):
            raise TypeError("NoLoCo state_dict has wrong shape")
        self._snapshot, self._m, self._v = (list(state[k]) for k in ("snapshot", "m", "v"))  # type: ignore[arg-type]
        self._inner_count = int(state.get("inner_count", 0))  # type: ignore[arg-type]
        self._step = int(state.get("step", 0))  # type: ignore[arg-type]


__all__ = ["AllReduceReducer", "DiLoCo", "DiLoCoConfig", "IdentityReducer", "NoLoCo", "NoLoCoConfig", "PeerReducer",
           "PseudoGradientReducer", "RingAllReduceSimulator", "ring_all_reduce", "ring_log2_rounds"]

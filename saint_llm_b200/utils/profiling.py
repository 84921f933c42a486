"""Profiling helpers (the reference has none).

* ``nvtx_range(name)``: an NVTX range around a region when ``SV4_NVTX=1`` (a no-op
  otherwise, so production code can keep the annotations);
* ``annotate_blocks(model)``: forward / backward NVTX ranges per transformer block and per
  attention / MoE module, through module hooks;
* ``DeviceTimer``: CUDA-event timing on the launching stream, synchronised on both sides,
  reported as the max over the ranks of a process group;
* ``PhaseRecorder``: named CUDA-event spans on the current stream (forward, backward,
  each expert-parallel stage, gradient sync, optimizer ...) summed per name and reported
  as the max over ranks; recording happens only while a recorder is active, so the
  instrumented code paths cost one global lookup otherwise;
* ``mfu``: model FLOP utilisation of a training step against a peak.
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Iterator

import torch
import torch.distributed as dist
from torch import nn


def nvtx_enabled() -> bool:
    return os.environ.get("SV4_NVTX", "0") not in ("", "0") and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not nvtx_enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def annotate_blocks(model: nn.Module) -> int:
    """Register NVTX push/pop hooks on every block and its attention / MoE submodules
    (forward and backward).  Returns the number of annotated modules; 0 when disabled."""
    if not nvtx_enabled():
        return 0
    n = 0
    for i, block in enumerate(getattr(model, "blocks", [])):
        for name, mod in (("block", block), ("attention", getattr(block, "attention", None)),
                          ("moe", getattr(block, "moe", None))):
            if mod is None:
                continue
            tag = f"L{i}.{name}"
            mod.register_forward_pre_hook(lambda m, a, t=tag: torch.cuda.nvtx.range_push(f"fwd:{t}"))
            mod.register_forward_hook(lambda m, a, o: torch.cuda.nvtx.range_pop())
            mod.register_full_backward_pre_hook(lambda m, g, t=tag: torch.cuda.nvtx.range_push(f"bwd:{t}"))
            mod.register_full_backward_hook(lambda m, gi, go: torch.cuda.nvtx.range_pop())
            n += 1
    return n


class DeviceTimer:
    """``with DeviceTimer(group) as t: ...``; ``t.ms`` is the device time of the region, max
    over the ranks of ``group`` (single process: its own)."""

    def __init__(self, group: dist.ProcessGroup | None = None, device: torch.device | None = None) -> None:
        self.group = group
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.ms = 0.0

    def __enter__(self) -> DeviceTimer:
        torch.cuda.synchronize(self.device)
        self._start = torch.cuda.Event(enable_timing=True)
        self._end = torch.cuda.Event(enable_timing=True)
        self._start.record()
        return self

    def __exit__(self, *exc: object) -> None:
        self._end.record()
        torch.cuda.synchronize(self.device)
        t = torch.tensor([self._start.elapsed_time(self._end)], device=self.device)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        self.ms = float(t.item())


class PhaseRecorder:
    """Per-phase device time of one (or a few) training steps.

    ``with PhaseRecorder(device) as rec: step()`` then ``rec.summary(group)`` returns
    ``{phase: ms}`` summed over every span of that phase, max over the ranks of ``group``.
    Instrumented code calls ``phase("name")`` (a context manager); spans of the same name
    add up, spans may nest (an outer "backward" contains the inner expert-parallel stages).
    Every rank must record the same phase names for the max-reduction to line up; the
    summary handles missing names by reducing over the sorted union gathered on the host."""

    _active: PhaseRecorder | None = None

    def __init__(self, device: torch.device | None = None) -> None:
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.spans: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def __enter__(self) -> PhaseRecorder:
        PhaseRecorder._active = self
        return self

    def __exit__(self, *exc: object) -> None:
        PhaseRecorder._active = None

    def summary(self, group: dist.ProcessGroup | None = None) -> dict[str, float]:
        torch.cuda.synchronize(self.device)
        tot: dict[str, float] = {}
        for name, a, b in self.spans:
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
        if dist.is_available() and dist.is_initialized():
            names: list = [None] * dist.get_world_size(group)
            dist.all_gather_object(names, sorted(tot), group=group)
            keys = sorted(set().union(*map(set, names)))
            t = torch.tensor([tot.get(k, 0.0) for k in keys], dtype=torch.float64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            tot = dict(zip(keys, t.tolist(), strict=True))
        return {k: round(v, 3) for k, v in sorted(tot.items())}


@contextlib.contextmanager
def phase(name: str) -> Iterator[None]:
    """A named span on the current CUDA stream while a ``PhaseRecorder`` is active."""
    rec = PhaseRecorder._active
    if rec is None:
        yield
        return
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    try:
        yield
    finally:
        b.record()
        rec.spans.append((name, a, b))


def mfu(tokens_per_s: float, active_params: float, peak_flops: float, *, attn_flops_per_token: float = 0.0) -> float:
    """6 N (+ attention) FLOPs per trained token over the peak (both per GPU or both per job)."""
    return tokens_per_s * (6.0 * active_params + attn_flops_per_token) / peak_flops


__all__ = ["DeviceTimer", "PhaseRecorder", "annotate_blocks", "mfu", "nvtx_enabled", "nvtx_range", "phase"]

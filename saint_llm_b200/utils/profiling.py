"""Profiling helpers (the reference has none).

* ``nvtx_range(name)``: an NVTX range around a region when ``SV4_NVTX=1`` (a no-op
  otherwise, so production code can keep the annotations);
* ``annotate_blocks(model)``: forward / backward NVTX ranges per transformer block and per
  attention / MoE module, through module hooks;
* ``DeviceTimer``: CUDA-event timing on the launching stream, synchronised on both sides,
  reported as the max over the ranks of a process group;
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


def mfu(tokens_per_s: float, active_params: float, peak_flops: float, *, attn_flops_per_token: float = 0.0) -> float:
    """6 N (+ attention) FLOPs per trained token over the peak (both per GPU or both per job)."""
    return tokens_per_s * (6.0 * active_params + attn_flops_per_token) / peak_flops


__all__ = ["DeviceTimer", "annotate_blocks", "mfu", "nvtx_enabled", "nvtx_range"]

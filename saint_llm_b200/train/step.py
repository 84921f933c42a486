"""``TrainStep``: the public one-call training step of the CUDA engine.

``step = TrainStep(model, optimizer, micro_batches=32, params=...)``;
``loss = step(host_tokens)`` copies the step's token batch from (pinned) host memory
to the GPU, runs forward / backward over the micro-batches with fp32 gradient
accumulation, applies the optimizer and returns the mean loss as a Python float
(one device->host read).  ``step.run_device(device_tokens)`` is the same step without
the copies and the read (used for device-side timing).
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor, nn

from saint_llm_b200.train.engine import zero_main_grads
from saint_llm_b200.utils.profiling import phase
from saint_llm_b200.train.losses import make_loss_fn


class TrainStep:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, micro_batches: int,
                 params: list[Tensor], loss_fn: nn.Module | None = None,
                 grad_sync: Callable[[list[Tensor]], None] | None = None) -> None:
        self.model = model
        self.optimizer = optimizer
        self.micro_batches = micro_batches
        self.params = params
        cfg = getattr(model, "cfg", None)
        self.loss_fn = loss_fn or make_loss_fn(cfg.mtp if cfg else None, moe_cfg=cfg.moe if cfg else None)
        self.grad_sync = grad_sync
        self.device = next(model.parameters()).device

    def run_device(self, tokens: Tensor) -> Tensor:
        """tokens: (micro_batches, mb, T) on the device.  Returns the mean loss (device scalar)."""
        self.model.train()
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        last_hook = getattr(self.grad_sync, "before_last_backward", None)
        for i in range(self.micro_batches):
            with phase("forward"):
                loss = self.loss_fn(self.model, tokens[i]) / self.micro_batches
            if last_hook is not None and i == self.micro_batches - 1:
                last_hook()
            with phase("backward"):
                loss.backward()
            total += loss.detach()
        if self.grad_sync is not None:
            with phase("grad_sync"):
                self.grad_sync(self.params)
        with phase("optimizer"):
            self.optimizer.step()
        post = getattr(self.grad_sync, "post_step", None)
        if post is not None:
            with phase("param_sync"):
                post()
        zero_main_grads(self.params)
        return total

    def __call__(self, host_tokens: Tensor) -> float:
        return float(self.run_device(host_tokens.to(self.device, non_blocking=True)).item())


__all__ = ["TrainStep"]

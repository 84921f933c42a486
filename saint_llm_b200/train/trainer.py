"""``Trainer``: a loop-level driver with loss-skip rules, gradient accumulation, clipping,
LR scheduling, metrics and checkpoint hooks.

Behaviour contract kept from the reference (``training/trainer.py:45-288``): a call of
``train_step(batch)`` is one micro-step and returns its loss as a float; every
``gradient_accumulation_steps`` accepted micro-steps make one optimizer step (clip ->
step -> scheduler tick -> metrics callback with ``loss``, ``lr`` and, when clipping,
``grad_norm``).  A micro-step whose loss is non-finite, or above ``loss_spike_factor``
times the median of the last ``loss_spike_window`` step losses (once at least four are
known), is a *skip*: the accumulated gradients are dropped, the accumulation window
restarts, and the callback gets ``skipped`` and ``skip_reason_<nan|spike>``.

The structure is this framework's own:

* ``SkipRule`` holds the loss history and decides; it works on host floats or, for a
  whole window at once, on a device tensor of losses.
* ``train_window(batches)`` is the fast path for the CUDA engine: all micro-steps of an
  accumulation window run back to back with their losses kept on the device, and the
  window costs ONE host read (the loss vector) before the optimizer step.  A skip inside a
  window drops the whole window (its gradients cannot be split after the fact).
* ``train_step(batch)`` keeps the per-micro-step contract (one host read per call, which
  the float return value needs).
* ``perf/step_s`` and ``perf/tokens_per_s`` are added to the metrics of every optimizer
  step.
"""

from __future__ import annotations

import math
import statistics
import time
from collections import deque
from collections.abc import Callable, Iterable, Sequence
from pathlib import Path
from typing import Any, Literal, Protocol

import torch
from torch import Tensor, nn

from saint_llm_b200.train.checkpoint import load_checkpoint, save_checkpoint

MixedPrecision = Literal["none", "bf16", "fp16"]
LossFn = Callable[[nn.Module, Tensor], Tensor]
MetricsCallback = Callable[[int, dict[str, float]], None]


class SchedulerLike(Protocol):
    def step(self) -> None: ...

    def state_dict(self) -> dict[str, Any]: ...

    def load_state_dict(self, state: dict[str, Any]) -> None: ...


class SkipRule:
    """Decides whether a loss value skips the update.

    ``nonfinite``: NaN / inf losses skip.  ``spike_factor``: a loss above factor x the
    median of the accepted history (``window`` most recent step losses, at least four)
    skips."""

    MIN_HISTORY = 4

    def __init__(self, *, nonfinite: bool, spike_factor: float | None, window: int) -> None:
        self.nonfinite = nonfinite
        self.spike_factor = spike_factor
        self.history: deque[float] = deque(maxlen=window)

    def threshold(self) -> float | None:
        if self.spike_factor is None or len(self.history) < self.MIN_HISTORY:
            return None
        return statistics.median(self.history) * self.spike_factor

    def reason(self, value: float) -> str | None:
        if self.nonfinite and not math.isfinite(value):
            return "nan"
        thr = self.threshold()
        if thr is not None and value > thr:
            return "spike"
        return None

    def reasons_device(self, losses: Tensor) -> Tensor:
        """Per-entry codes for a device vector of losses: 0 keep, 1 nan, 2 spike (no sync)."""
        codes = torch.zeros_like(losses, dtype=torch.int8)
        thr = self.threshold()
        if thr is not None:
            codes = torch.where(losses > thr, torch.full_like(codes, 2), codes)
        if self.nonfinite:
            codes = torch.where(~torch.isfinite(losses), torch.ones_like(codes), codes)
        return codes

    def accept(self, value: float) -> None:
        self.history.append(value)


def _check_args(grad_clip_norm, loss_spike_factor, loss_spike_window, accumulation, mixed_precision) -> None:
    problems = [
        (grad_clip_norm is not None and not grad_clip_norm > 0, f"grad_clip_norm={grad_clip_norm!r}: use None or > 0"),
        (loss_spike_factor is not None and not loss_spike_factor > 1.0,
         f"loss_spike_factor={loss_spike_factor!r}: use None or > 1"),
        (not loss_spike_window > 0, f"loss_spike_window={loss_spike_window!r}: needs at least one entry"),
        (not accumulation > 0, f"gradient_accumulation_steps={accumulation!r}: needs at least one micro-step"),
        (mixed_precision not in ("none", "bf16", "fp16"),
         f"mixed_precision={mixed_precision!r}: expected 'none', 'bf16' or 'fp16'"),
    ]
    bad = [msg for cond, msg in problems if cond]
    if bad:
        raise ValueError("invalid Trainer settings: " + "; ".join(bad))


class Trainer:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, loss_fn: LossFn,
                 lr_scheduler: SchedulerLike | None = None, grad_clip_norm: float | None = None,
                 metrics_callback: MetricsCallback | None = None, skip_nonfinite_loss: bool = True,
                 loss_spike_factor: float | None = None, loss_spike_window: int = 32,
                 gradient_accumulation_steps: int = 1, mixed_precision: MixedPrecision = "none",
                 device: torch.device | str | None = None) -> None:
        _check_args(grad_clip_norm, loss_spike_factor, loss_spike_window, gradient_accumulation_steps,
                    mixed_precision)
        self.model, self.optimizer, self.loss_fn = model, optimizer, loss_fn
        self.lr_scheduler = lr_scheduler
        self.grad_clip_norm = grad_clip_norm
        self.metrics_callback = metrics_callback
        self.gradient_accumulation_steps = gradient_accumulation_steps
        self.mixed_precision = mixed_precision
        self.rule = SkipRule(nonfinite=skip_nonfinite_loss, spike_factor=loss_spike_factor, window=loss_spike_window)
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.step = 0
        self.skipped_steps = 0
        self._pending = 0  # accepted micro-steps in the current window
        self._clock = (time.perf_counter(), 0)  # (time of the last step, tokens since)
        use_scaler = mixed_precision == "fp16" and self.device.type == "cuda"
        self._scaler = torch.amp.GradScaler(self.device.type) if use_scaler else None

    # ---------------------------------------------------------------- settings views
    @property
    def skip_nonfinite_loss(self) -> bool:
        return self.rule.nonfinite

    @property
    def loss_spike_factor(self) -> float | None:
        return self.rule.spike_factor

    # ---------------------------------------------------------------- pieces
    def _loss(self, batch: Tensor) -> Tensor:
        if self.mixed_precision == "none" or self.device.type != "cuda":
            return self.loss_fn(self.model, batch)
        dtype = {"bf16": torch.bfloat16, "fp16": torch.float16}[self.mixed_precision]
        with torch.amp.autocast(device_type="cuda", dtype=dtype):
            return self.loss_fn(self.model, batch).float()

    def _backward(self, loss: Tensor) -> None:
        k = self.gradient_accumulation_steps
        scaled = loss / k if k > 1 else loss
        (self._scaler.scale(scaled) if self._scaler is not None else scaled).backward()

    def _drop_window(self) -> None:
        self.optimizer.zero_grad(set_to_none=True)
        self._pending = 0

    def _report(self, metrics: dict[str, float]) -> None:
        if self.metrics_callback is not None:
            self.metrics_callback(self.step, metrics)

    def _skip(self, value: float, reason: str) -> None:
        self._drop_window()
        self.skipped_steps += 1
        self._report({"loss": value, "lr": self._lr(), "skipped": 1.0, f"skip_reason_{reason}": 1.0})

    def _lr(self) -> float:
        return float(self.optimizer.param_groups[0]["lr"])

    def _apply_update(self, value: float) -> None:
        """Clip, step, schedule and report once a window is complete."""
        if self._scaler is not None:
            self._scaler.unscale_(self.optimizer)
        metrics: dict[str, float] = {"loss": value, "lr": self._lr()}
        if self.grad_clip_norm is not None:
            metrics["grad_norm"] = float(torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.grad_clip_norm))
        if self._scaler is not None:
            self._scaler.step(self.optimizer)
            self._scaler.update()
        else:
            self.optimizer.step()
        self.optimizer.zero_grad()
        if self.lr_scheduler is not None:
            self.lr_scheduler.step()
        self.step += 1
        self._pending = 0
        self.rule.accept(value)
        t_prev, tokens = self._clock
        now = time.perf_counter()
        if now > t_prev and tokens:
            metrics["perf/step_s"] = now - t_prev
            metrics["perf/tokens_per_s"] = tokens / (now - t_prev)
        self._clock = (now, 0)
        self._report(metrics)

    def _count_tokens(self, batch: Tensor) -> None:
        t, n = self._clock
        self._clock = (t, n + batch.numel())

    # ---------------------------------------------------------------- public loop API
    def train_step(self, batch: Tensor) -> float:
        """One micro-step; returns its loss (one host read)."""
        self.model.train()
        batch = batch.to(self.device, non_blocking=True)
        self._count_tokens(batch)
        if self._pending == 0:
            self.optimizer.zero_grad()
        loss = self._loss(batch)
        value = float(loss.detach())
        reason = self.rule.reason(value)
        if reason is not None:
            self._skip(value, reason)
            return value
        self._backward(loss)
        self._pending += 1
        if self._pending == self.gradient_accumulation_steps:
            self._apply_update(value)
        return value

    def train_window(self, batches: Sequence[Tensor]) -> list[float]:
        """A whole accumulation window (``gradient_accumulation_steps`` micro-batches) with
        one host read: losses stay on the device until the optimizer decision."""
        k = self.gradient_accumulation_steps
        if len(batches) != k:
            raise ValueError(f"train_window takes exactly {k} micro-batches (got {len(batches)})")
        if self._pending:
            raise RuntimeError("train_window cannot start inside a window opened by train_step")
        self.model.train()
        self.optimizer.zero_grad()
        losses = torch.empty(k, dtype=torch.float32, device=self.device)
        for i, b in enumerate(batches):
            b = b.to(self.device, non_blocking=True)
            self._count_tokens(b)
            loss = self._loss(b)
            losses[i] = loss.detach().float()
            self._backward(loss)
        codes = self.rule.reasons_device(losses)
        host = torch.stack([losses, codes.float()]).tolist()  # the window's only host read
        values, flags = host[0], [int(c) for c in host[1]]
        bad = next((i for i, c in enumerate(flags) if c), None)
        if bad is not None:
            self._skip(values[bad], "nan" if flags[bad] == 1 else "spike")
            return values
        self._pending = k
        self._apply_update(values[-1])
        return values

    @torch.no_grad()
    def evaluate(self, eval_iter: Iterable[Tensor]) -> float:
        """Mean loss over ``eval_iter`` in eval mode (the previous mode is restored)."""
        was_training = self.model.training
        self.model.eval()
        try:
            vals = [self.loss_fn(self.model, b.to(self.device)).detach() for b in eval_iter]
        finally:
            self.model.train(was_training)
        if not vals:
            raise ValueError("evaluate() needs at least one batch")
        return float(torch.stack([v.float() for v in vals]).mean())

    # ---------------------------------------------------------------- checkpoints
    def save(self, path: str | Path, *, extra: dict[str, Any] | None = None) -> None:
        payload = dict(extra or {})
        if self.lr_scheduler is not None:
            payload["lr_scheduler"] = self.lr_scheduler.state_dict()
        save_checkpoint(path, self.model, self.optimizer, step=self.step, extra=payload)

    def load(self, path: str | Path, *, strict: bool = True) -> dict[str, Any]:
        meta = load_checkpoint(path, self.model, self.optimizer, strict=strict)
        self.step = int(meta.get("step", 0))
        extra = dict(meta.get("extra") or {})
        sched_state = extra.pop("lr_scheduler", None)
        if self.lr_scheduler is not None and sched_state is not None:
            self.lr_scheduler.load_state_dict(sched_state)
        return extra


__all__ = ["SkipRule", "Trainer"]

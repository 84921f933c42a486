"""``Trainer``: the reference's step semantics (``training/trainer.py:45-288``).

``train_step(batch)`` runs one micro-step: forward (optional CUDA autocast), loss,
non-finite / spike skip (median of the last ``loss_spike_window`` losses x factor,
needs >= 4), loss / K for accumulation, backward, and on the K-th micro-step grad
clip, optimizer step, scheduler tick and the metrics callback
``{loss, lr, grad_norm?, skipped?, skip_reason_*?}``.

The bench harness (``bench.py``) drives the model directly so that its timed
region has no per-micro-step host sync; this class keeps the reference's contract.
"""

from __future__ import annotations

import math
import time
from collections import deque
from collections.abc import Callable, Iterable
from pathlib import Path
from typing import Any, Literal, Protocol

import torch
from torch import Tensor, nn

from saint_llm_b200.train.checkpoint import load_checkpoint, save_checkpoint

MixedPrecision = Literal["none", "bf16", "fp16"]
LossFn = Callable[[nn.Module, Tensor], Tensor]
MetricsCallback = Callable[[int, dict[str, float]], None]


class _LRSchedulerLike(Protocol):
    def step(self) -> None: ...

    def state_dict(self) -> dict[str, Any]: ...

    def load_state_dict(self, state: dict[str, Any]) -> None: ...


class Trainer:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, loss_fn: LossFn,
                 lr_scheduler: _LRSchedulerLike | None = None, grad_clip_norm: float | None = None,
                 metrics_callback: MetricsCallback | None = None, skip_nonfinite_loss: bool = True,
                 loss_spike_factor: float | None = None, loss_spike_window: int = 32,
                 gradient_accumulation_steps: int = 1, mixed_precision: MixedPrecision = "none",
                 device: torch.device | str | None = None) -> None:
        if grad_clip_norm is not None and grad_clip_norm <= 0:
            raise ValueError(f"grad_clip_norm must be > 0 when set; got {grad_clip_norm}")
        if loss_spike_factor is not None and loss_spike_factor <= 1.0:
            raise ValueError(f"loss_spike_factor must be > 1.0 when set; got {loss_spike_factor}")
        if loss_spike_window <= 0:
            raise ValueError(f"loss_spike_window must be > 0; got {loss_spike_window}")
        if gradient_accumulation_steps <= 0:
            raise ValueError(f"gradient_accumulation_steps must be > 0; got {gradient_accumulation_steps}")
        if mixed_precision not in ("none", "bf16", "fp16"):
            raise ValueError(f"mixed_precision must be one of 'none' | 'bf16' | 'fp16'; got {mixed_precision!r}")
        self.model = model
        self.optimizer = optimizer
        self.loss_fn = loss_fn
        self.lr_scheduler = lr_scheduler
        self.grad_clip_norm = grad_clip_norm
        self.metrics_callback = metrics_callback
        self._t_last, self._tokens_since = time.perf_counter(), 0  # perf/ metrics
        self.skip_nonfinite_loss = skip_nonfinite_loss
        self.loss_spike_factor = loss_spike_factor
        self.gradient_accumulation_steps = gradient_accumulation_steps
        self.mixed_precision = mixed_precision
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.step = 0
        self.skipped_steps = 0
        self._recent_losses: deque[float] = deque(maxlen=loss_spike_window)
        self._micro_step = 0
        self._grad_scaler = (torch.amp.GradScaler(self.device.type)
                             if mixed_precision == "fp16" and self.device.type == "cuda" else None)

    # ------------------------------------------------------------------------------
    def _forward(self, batch: Tensor) -> Tensor:
        if self.mixed_precision == "none" or self.device.type != "cuda":
            return self.loss_fn(self.model, batch)
        dt = torch.bfloat16 if self.mixed_precision == "bf16" else torch.float16
        with torch.amp.autocast(device_type="cuda", dtype=dt):
            loss = self.loss_fn(self.model, batch)
        return loss.float()

    _forward_under_autocast = _forward

    def _is_loss_spike(self, value: float) -> bool:
        if self.loss_spike_factor is None or len(self._recent_losses) < 4:
            return False
        s = sorted(self._recent_losses)
        n = len(s)
        med = s[n // 2] if n % 2 else 0.5 * (s[n // 2 - 1] + s[n // 2])
        return value > med * self.loss_spike_factor

    def _fire(self, loss_value: float, *, grad_norm: float | None, skip_reason: str | None) -> None:
        if self.metrics_callback is None:
            return
        m: dict[str, float] = {"loss": loss_value, "lr": float(self.optimizer.param_groups[0]["lr"])}
        if grad_norm is not None:
            m["grad_norm"] = grad_norm
        if skip_reason is not None:
            m["skipped"] = 1.0
            m[f"skip_reason_{skip_reason}"] = 1.0
        else:
            now = time.perf_counter()
            dt = now - self._t_last
            if dt > 0 and self._tokens_since:
                m["perf/step_s"] = dt
                m["perf/tokens_per_s"] = self._tokens_since / dt
            self._t_last, self._tokens_since = now, 0
        self.metrics_callback(self.step, m)

    def train_step(self, batch: Tensor) -> float:
        self.model.train()
        batch = batch.to(self.device, non_blocking=True)
        self._tokens_since += batch.numel()
        loss = self._forward(batch)
        value = float(loss.detach().item())
        reason = None
        if self.skip_nonfinite_loss and not math.isfinite(value):
            reason = "nan"
        elif self.loss_spike_factor is not None and self._is_loss_spike(value):
            reason = "spike"
        if reason is not None:
            self.optimizer.zero_grad(set_to_none=True)
            self.skipped_steps += 1
            self._micro_step = 0
            self._fire(value, grad_norm=None, skip_reason=reason)
            return value
        k = self.gradient_accumulation_steps
        scaled = loss / k if k > 1 else loss
        if k == 1:
            self.optimizer.zero_grad()
        if self._grad_scaler is not None:
            self._grad_scaler.scale(scaled).backward()
        else:
            scaled.backward()
        self._micro_step += 1
        if self._micro_step < k:
            return value
        if self._grad_scaler is not None:
            self._grad_scaler.unscale_(self.optimizer)
        grad_norm = None
        if self.grad_clip_norm is not None:
            total = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.grad_clip_norm)
            grad_norm = float(total)
        if self._grad_scaler is not None:
            self._grad_scaler.step(self.optimizer)
            self._grad_scaler.update()
        else:
            self.optimizer.step()
        if k > 1:
            self.optimizer.zero_grad()
        if self.lr_scheduler is not None:
            self.lr_scheduler.step()
        self.step += 1
        self._micro_step = 0
        self._recent_losses.append(value)
        self._fire(value, grad_norm=grad_norm, skip_reason=None)
        return value

    @torch.no_grad()
    def evaluate(self, eval_iter: Iterable[Tensor]) -> float:
        was = self.model.training
        self.model.eval()
        try:
            total, n = 0.0, 0
            for b in eval_iter:
                total += float(self.loss_fn(self.model, b.to(self.device)).item())
                n += 1
            if n == 0:
                raise ValueError("evaluate() received an empty iterator")
            return total / n
        finally:
            if was:
                self.model.train()

    def save(self, path: str | Path, *, extra: dict[str, Any] | None = None) -> None:
        merged = dict(extra) if extra is not None else {}
        if self.lr_scheduler is not None:
            merged["lr_scheduler"] = self.lr_scheduler.state_dict()
        save_checkpoint(path, self.model, self.optimizer, step=self.step, extra=merged)

    def load(self, path: str | Path, *, strict: bool = True) -> dict[str, Any]:
        meta = load_checkpoint(path, self.model, self.optimizer, strict=strict)
        self.step = int(meta.get("step", 0))
        extra = dict(meta.get("extra") or {})
        if self.lr_scheduler is not None and "lr_scheduler" in extra:
            self.lr_scheduler.load_state_dict(extra.pop("lr_scheduler"))
        return extra


__all__ = ["Trainer"]

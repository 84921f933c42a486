"""LR schedule, checkpoint rotation and the wandb metrics adapter.

* ``warmup_cosine_schedule`` (reference ``training/schedule.py:20-75``): linear
  warm-up from 1e-8 x peak, then cosine to ``min_lr_ratio * min(peak lrs)``.
* ``CheckpointRotator`` (reference ``training/rotation.py:21-74``): writes
  ``<stem>.step<N><suffix>`` and keeps the last ``keep_last_n``.
* ``WandbLogger`` (reference ``training/wandb_logger.py:28-97``): a
  ``metrics_callback``; keys without ``/`` are prefixed ``train/``; the wandb module
  is imported lazily and can be injected for tests.
"""

from __future__ import annotations

import contextlib
from collections import deque
from pathlib import Path
from typing import Any, Literal

from torch.optim import Optimizer
from torch.optim.lr_scheduler import CosineAnnealingLR, LinearLR, LRScheduler, SequentialLR


def warmup_cosine_schedule(optimizer: Optimizer, *, warmup_steps: int, total_steps: int,
                           min_lr_ratio: float = 0.1) -> LRScheduler:
    if warmup_steps < 0:
        raise ValueError(f"warmup_steps must be ≥ 0; got {warmup_steps}")
    if warmup_steps >= total_steps:
        raise ValueError(f"warmup_steps={warmup_steps} must be < total_steps={total_steps}")
    if not 0.0 <= min_lr_ratio <= 1.0:
        raise ValueError(f"min_lr_ratio must be in [0, 1]; got {min_lr_ratio}")
    peaks = [g["lr"] for g in optimizer.param_groups]
    eta_min = min(peaks) * min_lr_ratio if peaks else 0.0
    if warmup_steps == 0:
        return CosineAnnealingLR(optimizer, T_max=total_steps, eta_min=eta_min)
    return SequentialLR(optimizer, schedulers=[
        LinearLR(optimizer, start_factor=1.0e-8, end_factor=1.0, total_iters=warmup_steps),
        CosineAnnealingLR(optimizer, T_max=total_steps - warmup_steps, eta_min=eta_min),
    ], milestones=[warmup_steps])


class CheckpointRotator:
    def __init__(self, base_path: str | Path, *, keep_last_n: int | None = 3) -> None:
        if keep_last_n is not None and keep_last_n <= 0:
            raise ValueError(f"keep_last_n must be > 0 when set; got {keep_last_n}")
        self.base_path = Path(base_path)
        self.keep_last_n = keep_last_n
        self._saved: deque[Path] = deque()

    def _path_for_step(self, step: int) -> Path:
        return self.base_path.with_name(f"{self.base_path.stem}.step{step}{self.base_path.suffix}")

    def save(self, trainer: Any, *, step: int | None = None, extra: dict[str, Any] | None = None) -> Path:
        path = self._path_for_step(trainer.step if step is None else step)
        trainer.save(path, extra=extra)
        self._saved.append(path)
        while self.keep_last_n is not None and len(self._saved) > self.keep_last_n:
            with contextlib.suppress(FileNotFoundError):
                self._saved.popleft().unlink()
        return path

    @property
    def saved_paths(self) -> tuple[Path, ...]:
        return tuple(self._saved)


class WandbLogger:
    def __init__(self, *, project: str, run_name: str | None = None, config: dict[str, Any] | None = None,
                 mode: Literal["online", "offline", "disabled"] = "online", tags: list[str] | None = None,
                 wandb_module: Any | None = None) -> None:
        if mode not in ("online", "offline", "disabled"):
            raise ValueError(f"mode must be online/offline/disabled; got {mode!r}")
        if wandb_module is None:
            import wandb as wandb_module  # type: ignore[no-redef]
        self._wandb = wandb_module
        self.run = wandb_module.init(project=project, name=run_name, config=config or {}, mode=mode,
                                     tags=tags or [])

    @staticmethod
    def _key(k: str) -> str:
        return k if "/" in k else f"train/{k}"

    def __call__(self, step: int, metrics: dict[str, float]) -> None:
        self._wandb.log({self._key(k): v for k, v in metrics.items()}, step=step)

    def finish(self) -> None:
        fin = getattr(self.run, "finish", None)
        if callable(fin):
            fin()


__all__ = ["CheckpointRotator", "WandbLogger", "warmup_cosine_schedule"]

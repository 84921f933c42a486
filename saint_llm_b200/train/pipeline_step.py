"""One training step under pipeline and/or context parallelism (config 4's PP x CP layout):
the counterpart of ``train.step.TrainStep`` that ``train.launch.build_training`` returns when
``RunConfig.pp`` or ``RunConfig.cp`` is above 1.

Layout over ``pp x cp`` ranks: rank r is CP rank ``r % cp`` of pipeline rank ``r // cp``.
The pipeline group links the ranks with one CP index; the CP group holds one pipeline rank's
shards.  Each pipeline rank keeps only its own blocks (the others are dropped at build time).

A step: the micro-batches run through the 1F1B schedule (``parallel.pipeline``) or DualPipe-V
(``parallel.dualpipe``), every CP rank computing its shard of each sequence; the loss is the
main next-token CE plus the MTP heads (``parallel.cp.shard_loss``) plus the MoE balance term,
whose per-sequence statistics are pooled over the CP group (``parallel.cp.balance_over``),
so the objective is the single-process training loss; gradients are
summed over the CP group and the tied embedding's over its two pipeline ends; the
attention-logit telemetry is max-reduced over the CP group (MuonClip acts on the same
value on every shard); then the optimizer updates the parameters this rank holds.

Gradients accumulate in the parameters' ``.grad`` (the parameter dtype: fp32 parameters keep
fp32 sums; with bf16 parameters the micro-batch sums are bf16, unlike ``TrainStep``'s fp32
``main_grad`` buffers).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor, nn


class PipelineTrainStep:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, micro_batches: int,
                 pp_group: dist.ProcessGroup | None, cp_group: dist.ProcessGroup | None,
                 schedule: str = "1f1b", mtp: bool = True, stage: object | None = None,
                 group: dist.ProcessGroup | None = None) -> None:
        """``group``: all ``pp x cp`` ranks of the job (the default group when None)."""
        from saint_llm_b200.parallel.dualpipe import DualPipeV
        from saint_llm_b200.parallel.pipeline import PipelineStage

        if schedule not in ("1f1b", "dualpipe"):
            raise ValueError(f"unknown pipeline schedule {schedule!r}")
        self.model, self.optimizer = model, optimizer
        self.micro_batches, self.schedule, self.mtp = micro_batches, schedule, mtp
        self.cp_group, self.group = cp_group, group
        self.device = next(model.parameters()).device
        if stage is not None:
            self.stage = stage
        elif schedule == "dualpipe":
            self.stage = DualPipeV(model, pp_group, prune=True, cp_group=cp_group)
        else:
            self.stage = PipelineStage(model, pp_group, prune=True, cp_group=cp_group)

    def _loss(self, model: nn.Module, h: Tensor, ids: Tensor) -> Tensor:
        from saint_llm_b200.parallel.cp import shard_loss

        r = dist.get_rank(self.cp_group) if self.cp_group is not None else 0
        return shard_loss(model, h, ids, r * h.shape[1], mtp=self.mtp)

    @torch.no_grad()
    def _sync_logits(self) -> None:
        if self.cp_group is None:
            return
        bufs = [m.max_attn_logit for m in self.model.modules()
                if isinstance(getattr(m, "max_attn_logit", None), Tensor)]
        if bufs:
            flat = torch.stack([b.float() for b in bufs])
            dist.all_reduce(flat, op=dist.ReduceOp.MAX, group=self.cp_group)
            for b, v in zip(bufs, flat, strict=True):
                b.copy_(v)

    def run_device(self, tokens: Tensor) -> Tensor:
        """tokens: (micro_batches, mb, T) on the device, the same on every rank.  Returns the
        step's mean main + MTP loss (device scalar, the same on every rank); the balance term
        is in the gradients but not in the reported value."""
        from saint_llm_b200.parallel.dualpipe import run_dualpipe
        from saint_llm_b200.parallel.pipeline import run_1f1b, sync_cp_grads, sync_tied_embedding

        self.model.train()
        micro = [tokens[i] for i in range(tokens.shape[0])]
        aux_w = float(self.model.cfg.moe.sequence_balance_weight)  # type: ignore[attr-defined]
        if self.schedule == "dualpipe":
            out = run_dualpipe(self.stage, micro, loss_fn=self._loss, aux_weight=aux_w)  # type: ignore[arg-type]
        else:
            out = run_1f1b(self.stage, micro, loss_fn=self._loss, aux_weight=aux_w)  # type: ignore[arg-type]
            sync_tied_embedding(self.stage)  # type: ignore[arg-type]
        sync_cp_grads(self.stage)  # type: ignore[arg-type]
        self._sync_logits()
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        # the loss lives on the CP ranks of the last stage (DualPipe-V: of pipeline rank 0) as
        # shares; the sum over every rank is the step's loss
        total = (out.detach().float().reshape(()) if out is not None
                 else torch.zeros((), dtype=torch.float32, device=self.device)).clone()
        if dist.is_initialized():
            dist.all_reduce(total, group=self.group)
        return total

    def __call__(self, host_tokens: Tensor) -> float:
        return float(self.run_device(host_tokens.to(self.device, non_blocking=True)).item())


__all__ = ["PipelineTrainStep"]

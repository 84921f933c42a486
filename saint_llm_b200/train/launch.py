"""Build a training job from a ``ModelConfig`` (what the model is) and a ``RunConfig`` (how
it runs): the public entry point behind ``bench.py`` and user scripts.

    job = build_training(model_cfg, run_cfg, device)
    loss = job.step(host_tokens)          # (grad_accum, micro_batch, seq_len) int64

What each ``RunConfig`` field selects here:

* ``ep`` / ``zero``: ``ep > 1`` shards the routed experts over the process group (EP must
  equal the world size, one node); ``zero="hybrid_zero"`` gives every replicated
  parameter one owner that reduces, updates and broadcasts it, ``"dp"`` all-reduces the
  replicated gradients and updates them everywhere.
* ``fused_ep``: the expert-parallel token traffic runs in this framework's peer-memory
  kernels (True) or over NCCL ``all_to_all`` (False, the baseline and oracle).
* ``fused_zero``: with hybrid ZeRO, each transformer block's per-owner gradient reductions
  are issued from a backward hook during the step's last micro-batch, so they run on
  NCCL's stream while the backward of the earlier blocks continues (True), or all after
  the backward (False).
* ``zero_transport``: with hybrid ZeRO, NCCL ``reduce`` / ``broadcast`` ("nccl"), this
  framework's peer-memory pull kernels ("p2p", ``parallel.zero_p2p``), or "auto" (p2p on CUDA).
* ``cuda_graphs``: on one GPU, each micro-batch's forward + backward replays one captured
  CUDA graph (``TrainStep(cuda_graph=True)``); ignored when gradients are synchronised
  across ranks (the expert-parallel step reads routing sizes on the host).
* ``fp8_expert_cache``: with ``linear_quant="fp8"``, whether the routed experts' FP8 weight
  copies persist between steps (set on every expert pool as ``fp8_weight_cache``).
* ``kernels``: "native" (sm_100a kernels) or "torch" (the eager oracle path on CUDA,
  through ``backend.eager_mode``; every step then runs inside that mode).
* ``micro_batch`` / ``seq_len`` / ``grad_accum``: the shape of one step's token batch.
* ``lr`` / ``adamw_lr``: Muon and AdamW learning rates.
* ``pg_timeout_s``: the process-group timeout (used when this function initialises it);
  ``device_wait_timeout_ms``: the bound of every cross-GPU flag wait of the EP kernels.
* ``seed``: the model initialisation seed.
* ``param_dtype`` / ``grad_dtype`` / ``compute_dtype``: parameters in bf16 (or fp32),
  gradients accumulated in fp32 ``main_grad`` buffers; bf16 parameters compute in bf16.
  Other combinations raise.
* ``tp``: attention heads sharded over groups of ``tp`` consecutive ranks, composed with EP over
  the whole group and (hybrid ZeRO) data parallelism over the ``world / tp`` replicas
  (``parallel.tp_ep``); the ranks of one TP group must be fed the same batch
  (``TrainingJob.replica`` names it).  ``fused_tp`` selects the peer-memory TP kernels.
* ``pp`` / ``cp`` (with ``ep = tp = 1``, ``world = pp x cp``): config 4's layout -- the block
  stack in ``pp`` pipeline stages (``pp_schedule``: 1F1B or DualPipe-V), each sequence split
  over the ``cp`` ranks of a stage; the step is ``train.pipeline_step.PipelineTrainStep``
  (main + MTP loss) and every rank reads the same batch.
"""

from __future__ import annotations

import contextlib
import datetime
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.distributed as dist
from torch import Tensor, nn

from saint_llm_b200.config import ModelConfig, RunConfig


@dataclass
class TrainingJob:
    model: nn.Module
    optimizer: torch.optim.Optimizer
    step: TrainStepLike
    grad_sync: object | None
    run: RunConfig
    # which shard of the global batch this rank reads, out of how many (ranks of one TP
    # group read the same shard)
    replica: int = 0
    replicas: int = 1

    def save(self, directory: str | Path, *, step: int, extra: dict | None = None) -> Path:
        """Sharded (v2) checkpoint, collective: every rank writes its optimizer state, rank 0
        the full unsharded model (``parallel.state.gather_full_state_dict``) and the manifest
        last, so a directory with a manifest is complete."""
        from saint_llm_b200.parallel.state import gather_full_state_dict
        from saint_llm_b200.train.checkpoint import save_sharded

        world, rank = _world_rank()
        if self.run.pp > 1 or self.run.cp > 1:
            from saint_llm_b200.parallel.state import gather_pipeline_state_dict

            full = gather_pipeline_state_dict(self.model, self.step.stage)  # type: ignore[attr-defined]
        else:
            full = gather_full_state_dict(self.model) if world > 1 else self.model.state_dict()
        opt_state = self.optimizer.state_dict()
        extra = {**(extra or {}), "layout": self._layout(world)}
        if rank != 0:
            save_sharded(directory, full, opt_state, step=step, rank=rank, world_size=world, extra=extra)
        if world > 1:
            dist.barrier()  # every optimizer shard is on disk before rank 0 writes the manifest
        if rank == 0:
            save_sharded(directory, full, opt_state, step=step, rank=0, world_size=world, extra=extra,
                         model_config_json=self.model.cfg.model_dump_json())  # type: ignore[union-attr]
        if world > 1:
            dist.barrier()
        return Path(directory)

    def load(self, directory: str | Path, *, optimizer: bool = True) -> int:
        """Resume from ``save``'s directory (or any v2 checkpoint): the full model state is
        sliced into this rank's shards; the optimizer state is restored when the checkpoint
        was written with the same layout (world size, TP, EP, ZeRO: its state is per rank and
        per shard) and skipped otherwise (fresh moments).  Returns the step."""
        from saint_llm_b200.ops.fp8 import bump_weight_epoch
        from saint_llm_b200.parallel.state import load_full_state_dict
        from saint_llm_b200.train.checkpoint import load_sharded

        world, rank = _world_rank()
        manifest = _manifest(directory)
        saved = (manifest.get("extra") or {}).get("layout")
        # optimizer states are per rank and per shard shape: only the same layout reuses them
        same_layout = saved == self._layout(world) if saved is not None else manifest["world_size"] == world
        data = load_sharded(directory, rank=rank if same_layout else 0)
        load_full_state_dict(self.model, data["model"])
        if optimizer and same_layout and data["optim"] is not None:
            self.optimizer.load_state_dict(data["optim"])
        bump_weight_epoch()  # cached FP8 weight copies must be re-quantised from the loaded weights
        return int(data["step"])

    def _layout(self, world: int) -> dict:
        return {"world": world, "tp": self.run.tp, "ep": self.run.ep, "zero": self.run.zero, "pp": self.run.pp,
                "cp": self.run.cp, "pp_schedule": self.run.pp_schedule}

    def close(self) -> None:
        """Collective release of the expert-parallel peer buffers (call on every rank)."""
        comm = getattr(self.model, "ep_comm", None)
        if comm is not None:
            comm.close()
        tp_comm = getattr(self.grad_sync, "tp_comm", None)
        if tp_comm is not None:
            tp_comm.close()


def _world_rank() -> tuple[int, int]:
    return (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)


def _manifest(directory: str | Path) -> dict:
    import json

    return json.loads((Path(directory) / "manifest.json").read_text())


class TrainStepLike:  # typing helper: TrainStep or its eager wrapper
    def __call__(self, host_tokens: Tensor) -> float: ...

    def run_device(self, tokens: Tensor) -> Tensor: ...


class _EagerStep:
    """Runs every call of a ``TrainStep`` under ``backend.eager_mode`` (kernels="torch")."""

    def __init__(self, inner) -> None:
        self.inner = inner

    def _ctx(self) -> contextlib.AbstractContextManager:
        from saint_llm_b200.ops import backend

        return backend.eager_mode(True)

    def __call__(self, host_tokens: Tensor) -> float:
        with self._ctx():
            return self.inner(host_tokens)

    def run_device(self, tokens: Tensor) -> Tensor:
        with self._ctx():
            return self.inner.run_device(tokens)

    def __getattr__(self, name: str):
        return getattr(self.inner, name)


def _check(run: RunConfig, world: int) -> None:
    problems = []
    if run.pp > 1 or run.cp > 1:
        if run.pp * run.cp != world:
            problems.append(f"pp x cp = {run.pp} x {run.cp} must equal the world size {world}")
        if run.ep != 1 or run.tp != 1:
            problems.append("pipeline / context parallelism runs with ep = tp = 1")
    if run.ep not in (1, world):
        problems.append(f"ep={run.ep} must be 1 or the world size {world}")
    if run.tp < 1 or world % run.tp:
        problems.append(f"tp={run.tp} must divide the world size {world}")
    elif run.tp > 1 and run.ep != world:
        problems.append(f"tp={run.tp} composes with expert parallelism over all ranks: ep must be {world}")
    if run.zero not in ("dp", "hybrid_zero", "none"):
        problems.append(f"zero={run.zero!r} (this builder runs 'dp' or 'hybrid_zero'; FSDP has parallel.fsdp)")
    if run.grad_dtype != "float32":
        problems.append("grad_dtype must be float32 (gradients accumulate in fp32 main_grad buffers)")
    if run.param_dtype == "bfloat16" and run.compute_dtype != "bfloat16":
        problems.append("bf16 parameters compute in bf16")
    if problems:
        raise ValueError("RunConfig not supported by build_training: " + "; ".join(problems))


def init_distributed(run: RunConfig, device: torch.device) -> None:
    """NCCL process group with the run's timeout (no-op when already initialised)."""
    if dist.is_initialized():
        return
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=run.pg_timeout_s), device_id=device)


def build_training(model_cfg: ModelConfig, run: RunConfig, device: torch.device, *,
                   group: dist.ProcessGroup | None = None, qk_clip: bool = True) -> TrainingJob:
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.train.engine import attach_main_grads, cast_params
    from saint_llm_b200.train.step import TrainStep

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    _check(run, world)
    torch.manual_seed(run.seed)
    with torch.device(device):
        model = SaintLLM(model_cfg)
    if run.param_dtype == "bfloat16":
        cast_params(model, torch.bfloat16)
    for mod in model.modules():
        if hasattr(mod, "gate_weight") and hasattr(mod, "linear_quant"):
            mod.fp8_weight_cache = run.fp8_expert_cache
    if run.pp > 1 or run.cp > 1:
        return _build_pipeline(model, run, group, qk_clip)
    grad_sync = None
    replica, replicas = (dist.get_rank(group), world) if world > 1 else (0, 1)
    if world > 1:
        common = dict(transport="p2p" if run.fused_ep else "nccl", zero=run.zero == "hybrid_zero",
                      timeout_s=run.device_wait_timeout_ms / 1000.0, overlap_reduce=run.fused_zero,
                      zero_transport=run.zero_transport)
        if run.tp > 1:
            from saint_llm_b200.parallel.tp_ep import setup_tp_ep

            grad_sync, lay = setup_tp_ep(model, run.tp, group, tp_transport="p2p" if run.fused_tp else "nccl",
                                         max_tokens=run.micro_batch * run.seq_len, **common)
            replica, replicas = lay.replica, lay.replicas
        else:
            from saint_llm_b200.parallel import ep as ep_mod

            grad_sync = ep_mod.setup_expert_parallel(model, group, **common)
        if device.type == "cuda":
            torch.cuda.empty_cache()
    params = attach_main_grads(model)
    muon, adamw = split_for_muon_adamw(model)
    opt = MuonAdamW(muon, adamw, lr=run.lr, adamw_lr=run.adamw_lr,
                    qk_clip_layers=model.attention_layers() if qk_clip else None)
    if grad_sync is not None:
        grad_sync.configure_optimizer(opt)
    step = TrainStep(model, opt, micro_batches=run.grad_accum, params=params, grad_sync=grad_sync,
                     cuda_graph=run.cuda_graphs and run.kernels == "native")
    wrapped = _EagerStep(step) if run.kernels == "torch" else step
    return TrainingJob(model, opt, wrapped, grad_sync, run, replica, replicas)


def pp_cp_groups(pp: int, cp: int, group: dist.ProcessGroup | None = None
                 ) -> tuple[dist.ProcessGroup | None, dist.ProcessGroup | None]:
    """(pipeline group, CP group) of this rank: rank r is CP rank r % cp of pipeline rank
    r // cp.  Every rank of ``group`` calls this (new groups are created collectively)."""
    rank = dist.get_rank(group)
    glob = [dist.get_global_rank(group, r) if group is not None else r for r in range(pp * cp)]
    pp_group = cp_group = None
    for c in range(cp):
        g = dist.new_group([glob[s * cp + c] for s in range(pp)])
        if rank % cp == c:
            pp_group = g
    for s in range(pp):
        g = dist.new_group([glob[s * cp + c] for c in range(cp)])
        if rank // cp == s:
            cp_group = g
    return pp_group, cp_group


def _build_pipeline(model: nn.Module, run: RunConfig, group: dist.ProcessGroup | None, qk_clip: bool) -> TrainingJob:
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.parallel.dualpipe import DualPipeV
    from saint_llm_b200.parallel.pipeline import PipelineStage
    from saint_llm_b200.train.pipeline_step import PipelineTrainStep

    pp_group, cp_group = pp_cp_groups(run.pp, run.cp, group)
    # the stage drops the other stages' blocks before the optimizer sees any parameter
    stage = (DualPipeV(model, pp_group, prune=True, cp_group=cp_group) if run.pp_schedule == "dualpipe"
             else PipelineStage(model, pp_group, prune=True, cp_group=cp_group))
    muon, adamw = split_for_muon_adamw(model)
    layers = [b.attention for b in model.blocks if hasattr(b, "attention")]  # type: ignore[attr-defined]
    opt = MuonAdamW(muon, adamw, lr=run.lr, adamw_lr=run.adamw_lr, qk_clip_enabled=qk_clip,
                    qk_clip_layers=layers if qk_clip else None)
    step = PipelineTrainStep(model, opt, micro_batches=run.grad_accum, pp_group=pp_group, cp_group=cp_group,
                             schedule=run.pp_schedule, stage=stage, group=group)
    return TrainingJob(model, opt, step, None, run, 0, 1)


__all__ = ["TrainingJob", "build_training", "init_distributed", "pp_cp_groups"]

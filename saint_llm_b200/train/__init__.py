"""Training layer: Trainer, losses, checkpoints (v1 + sharded v2), rotation, LR schedule,
wandb adapter, synthetic data and the training-step engine used by bench.py."""

from saint_llm_b200.train.checkpoint import (
    experts_to_per_module,
    experts_to_stacked,
    load_checkpoint,
    load_sharded,
    save_checkpoint,
    save_sharded,
    sharded_to_v1,
)
from saint_llm_b200.train.losses import cross_entropy_main, cross_entropy_with_mtp, make_loss_fn
from saint_llm_b200.train.schedule import CheckpointRotator, WandbLogger, warmup_cosine_schedule
from saint_llm_b200.train.trainer import Trainer

__all__ = [
    "CheckpointRotator",
    "Trainer",
    "WandbLogger",
    "cross_entropy_main",
    "cross_entropy_with_mtp",
    "experts_to_per_module",
    "experts_to_stacked",
    "load_checkpoint",
    "load_sharded",
    "make_loss_fn",
    "save_checkpoint",
    "save_sharded",
    "sharded_to_v1",
    "warmup_cosine_schedule",
]

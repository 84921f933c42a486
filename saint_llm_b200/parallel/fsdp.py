"""Process-group bootstrap and FSDP2 wrapping (reference: ``saint_llm_distributed/fsdp.py``):
an idempotent single-rank gloo group on 127.0.0.1 for local use, a 1-D device mesh, and
``fully_shard`` applied to every ``*Block`` submodule with trainable parameters, then the
root.  FSDP2 is kept as a baseline mode; the framework's own data/expert-parallel engine is
in ``parallel.ep`` and ``parallel.zero``."""

from __future__ import annotations

import os
from collections.abc import Callable

import torch.distributed as dist
from torch import nn

ShardPolicy = Callable[[str, nn.Module], bool]


def ensure_local_gloo_pg(*, master_addr: str = "127.0.0.1", master_port: str = "29500", rank: int = 0,
                         world_size: int = 1) -> bool:
    if dist.is_initialized():
        return False
    for k, v in (("MASTER_ADDR", master_addr), ("MASTER_PORT", master_port), ("WORLD_SIZE", str(world_size)),
                 ("RANK", str(rank))):
        os.environ.setdefault(k, v)
    dist.init_process_group(backend="gloo", world_size=world_size, rank=rank)
    return True


def init_default_mesh(*, device: str = "cpu", world_size: int | None = None):  # noqa: ANN201
    if not dist.is_initialized():
        raise RuntimeError("process group not initialized; call ensure_local_gloo_pg() or init_process_group first")
    return dist.device_mesh.init_device_mesh(device, (world_size or dist.get_world_size(),))


def default_block_policy(name: str, module: nn.Module) -> bool:
    return bool(name) and type(module).__name__.endswith("Block") and any(p.requires_grad for p in module.parameters())


def fsdp2_wrap(model: nn.Module, *, mesh=None, policy: ShardPolicy | None = None,  # noqa: ANN001
               wrap_root: bool = True) -> nn.Module:
    from torch.distributed.fsdp import fully_shard

    mesh = mesh if mesh is not None else init_default_mesh()
    policy = policy or default_block_policy
    for name, sub in model.named_modules():
        if name and policy(name, sub):
            fully_shard(sub, mesh=mesh)
    if wrap_root:
        fully_shard(model, mesh=mesh)
    return model


__all__ = ["ShardPolicy", "default_block_policy", "ensure_local_gloo_pg", "fsdp2_wrap", "init_default_mesh"]

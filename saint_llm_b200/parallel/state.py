"""Full (unsharded) state dicts of a model sharded by expert and/or tensor parallelism, and
the reverse: the bridge between a parallel run and the checkpoint formats of
``train.checkpoint``, whose model state is always the single-process state dict (so a run can
resume at another world size or layout, and the reference loads the file).

What is sharded, and how it is put back:

* routed experts (``parallel.ep.shard_grouped_experts``): ``*.moe.grouped_experts.*_weight``
  hold rank r's experts ``[r*E/N, (r+1)*E/N)`` of the layer's EP group -> concatenated along
  dim 0 in group-rank order;
* head-sharded attention (``parallel.tp.shard_attention_heads``): ``q_up.weight`` rows and
  ``sink_logit`` entries -> dim 0; ``output.final_proj.weight`` columns -> dim 1; the output
  groups ``output.group_projs.{i}`` of TP rank r are the full model's groups ``r*g/t + i``.

Every other tensor is replicated and taken from the local copy.  ``gather_full_state_dict``
is collective over the groups the model was sharded with (call it on every rank);
``load_full_state_dict`` is local.
"""

from __future__ import annotations

import re

import torch
import torch.distributed as dist
from torch import Tensor, nn

_GROUP_PROJ = re.compile(r"^(.*\.output)\.group_projs\.(\d+)\.(.+)$")


def _sharded_modules(model: nn.Module) -> tuple[dict[str, nn.Module], dict[str, nn.Module]]:
    """(prefix -> MoE layer with ep_size > 1, prefix -> attention module with a TP group)."""
    from saint_llm_b200.models.moe import DeepSeekMoE

    moes, attns = {}, {}
    for name, mod in model.named_modules():
        if isinstance(mod, DeepSeekMoE) and mod.ep_size > 1:
            moes[name] = mod
        if getattr(mod, "tp_group", None) is not None and hasattr(mod, "attn_cfg"):
            attns[name] = mod
    return moes, attns


def _all_gather(t: Tensor, group: dist.ProcessGroup | None) -> list[Tensor]:
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    return parts


def _attn_rule(key: str, attns: dict[str, nn.Module]) -> tuple[nn.Module, str] | None:
    """(attention module, the key relative to it) when ``key`` belongs to a TP-sharded one."""
    for prefix, mod in attns.items():
        if key.startswith(prefix + "."):
            return mod, key[len(prefix) + 1:]
    return None


@torch.no_grad()
def gather_full_state_dict(model: nn.Module, *, device: str | torch.device = "cpu") -> dict[str, Tensor]:
    """The state dict of the unsharded model, on ``device``, on every rank (collective)."""
    moes, attns = _sharded_modules(model)
    local = model.state_dict()
    full: dict[str, Tensor] = {}
    for key, t in local.items():
        moe = next((m for p, m in moes.items() if key.startswith(p + ".grouped_experts.")), None)
        rule = _attn_rule(key, attns)
        if moe is not None:
            full[key] = torch.cat([p.to(device) for p in _all_gather(t, moe.ep_group)], 0)
        elif rule is not None:
            mod, rel = rule
            g = mod.tp_group
            if rel in ("q_up.weight", "sink_logit"):
                full[key] = torch.cat([p.to(device) for p in _all_gather(t, g)], 0)
            elif rel == "output.final_proj.weight":
                full[key] = torch.cat([p.to(device) for p in _all_gather(t, g)], 1)
            elif (m := _GROUP_PROJ.match(key)) is not None:
                per = mod.output.n_groups
                for r, p in enumerate(_all_gather(t, g)):
                    full[f"{m.group(1)}.group_projs.{r * per + int(m.group(2))}.{m.group(3)}"] = p.to(device)
            else:
                full[key] = t.detach().to(device).clone()
        else:
            full[key] = t.detach().to(device).clone()
    return full


@torch.no_grad()
def load_full_state_dict(model: nn.Module, full: dict[str, Tensor], *, strict: bool = True) -> None:
    """Load an unsharded state dict into this rank's shards of ``model`` (the inverse of
    ``gather_full_state_dict``; no communication)."""
    moes, attns = _sharded_modules(model)
    local: dict[str, Tensor] = {}
    for key, t in model.state_dict().items():
        moe = next((m for p, m in moes.items() if key.startswith(p + ".grouped_experts.")), None)
        rule = _attn_rule(key, attns)
        if moe is not None:
            n = t.shape[0]
            local[key] = full[key][moe.ep_rank * n:(moe.ep_rank + 1) * n]
        elif rule is not None:
            mod, rel = rule
            r = dist.get_rank(mod.tp_group)
            if rel in ("q_up.weight", "sink_logit"):
                n = t.shape[0]
                local[key] = full[key][r * n:(r + 1) * n]
            elif rel == "output.final_proj.weight":
                n = t.shape[1]
                local[key] = full[key][:, r * n:(r + 1) * n]
            elif (m := _GROUP_PROJ.match(key)) is not None:
                local[key] = full[f"{m.group(1)}.group_projs.{r * mod.output.n_groups + int(m.group(2))}.{m.group(3)}"]
            elif key in full:
                local[key] = full[key]
        elif key in full:
            local[key] = full[key]
    model.load_state_dict(local, strict=strict)


@torch.no_grad()
def gather_pipeline_state_dict(model: nn.Module, stage: object) -> dict[str, Tensor]:
    """The full state dict of a model split into pipeline stages (``parallel.pipeline`` /
    ``parallel.dualpipe``, blocks of other stages dropped), on the CPU, on every rank
    (collective over the pipeline group).  Each block comes from the stage that holds it; the
    input embedding from the first stage, everything else outside the blocks (final norm, MTP
    heads, LM head) from the stage that computes the loss, which is where they are updated.
    ``load_full_state_dict`` loads the result back into any stage."""
    group = stage.group  # type: ignore[attr-defined]
    n = dist.get_world_size(group)
    mine = {k: v.detach().cpu() for k, v in model.state_dict().items()}
    parts: list = [None] * n
    dist.all_gather_object(parts, mine, group=group)
    dual = hasattr(stage, "bounds")  # DualPipe-V: both ends live on pipeline rank 0
    first, last = 0, (0 if dual else n - 1)
    full: dict[str, Tensor] = {}
    for r, sd in enumerate(parts):
        for k, v in sd.items():
            if k.startswith("blocks."):
                full.setdefault(k, v)
            elif k.startswith("embed.") and r == first:
                full[k] = v
            elif not k.startswith("embed.") and r == last:
                full[k] = v
    return full


__all__ = ["gather_full_state_dict", "gather_pipeline_state_dict", "load_full_state_dict"]

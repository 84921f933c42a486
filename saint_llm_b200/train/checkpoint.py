"""Checkpoints: the reference's single-file format (v1) and a sharded extension (v2).

v1 (reference ``training/checkpoint.py:21-85``) is one ``torch.save`` dict::

    {"format_version": 1, "step": int, "model": state_dict,
     "optimizer": state_dict | None, "extra": dict | None}

Files written by either framework load in the other (same state-dict keys).  Writes
here are atomic: the payload goes to ``<path>.tmp`` and is renamed into place, so a
process killed mid-save leaves the previous checkpoint intact.

v2 (sharded): a directory with ``manifest.json`` (format_version 2, step, world size,
model config, per-rank file list), ``model.pt`` (the full model state dict, written by
rank 0: ``parallel.state.gather_full_state_dict`` assembles it from expert- and
tensor-parallel shards, ``load_full_state_dict`` slices it back) and ``optim.rank{r}.pt``
per rank.
``load_sharded(..., into_v1=True)`` gathers everything back into the v1 layout so a
run can resume at a different world size.

Layout converters switch experts between the per-module layout
(``moe.routed_experts.{j}.{gate,up,down}_proj.weight``) and the stacked layout
(``moe.grouped_experts.{gate,up,down}_weight``).
"""

from __future__ import annotations

import json
import os
import re
from pathlib import Path
from typing import Any

import torch
from torch import Tensor, nn

FORMAT_V1 = 1
FORMAT_V2 = 2


def _atomic_save(obj: Any, path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def save_checkpoint(path: str | Path, model: nn.Module, optimizer: torch.optim.Optimizer | None = None, *,
                    step: int, extra: dict[str, Any] | None = None) -> None:
    _atomic_save({
        "format_version": FORMAT_V1,
        "step": int(step),
        "model": model.state_dict(),
        "optimizer": optimizer.state_dict() if optimizer is not None else None,
        "extra": dict(extra) if extra is not None else None,
    }, Path(path))


def load_checkpoint(path: str | Path, model: nn.Module, optimizer: torch.optim.Optimizer | None = None, *,
                    map_location: str | torch.device | None = None, strict: bool = True) -> dict[str, Any]:
    payload = torch.load(path, map_location=map_location, weights_only=False)
    if "model" not in payload:
        raise ValueError(f"checkpoint at {path} missing 'model' key")
    model.load_state_dict(payload["model"], strict=strict)
    if optimizer is not None:
        if payload.get("optimizer") is None:
            raise ValueError(f"checkpoint at {path} has no optimizer state but caller passed one")
        optimizer.load_state_dict(payload["optimizer"])
    return {"step": int(payload.get("step", 0)), "extra": payload.get("extra"),
            "format_version": int(payload.get("format_version", FORMAT_V1))}


# ------------------------------------------------------------------------ sharded (v2)
def save_sharded(directory: str | Path, model_state: dict[str, Tensor], optim_state: dict[str, Any] | None, *,
                 step: int, rank: int, world_size: int, model_config_json: str | None = None,
                 extra: dict[str, Any] | None = None) -> Path:
    """Each rank writes its optimizer shard; rank 0 writes the model and the manifest last."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    if optim_state is not None:
        _atomic_save(optim_state, d / f"optim.rank{rank}.pt")
    if rank == 0:
        _atomic_save(model_state, d / "model.pt")
        manifest = {
            "format_version": FORMAT_V2, "step": int(step), "world_size": int(world_size),
            "model": "model.pt", "optim": [f"optim.rank{r}.pt" for r in range(world_size)],
            "model_config": model_config_json, "extra": extra,
        }
        tmp = d / "manifest.json.tmp"
        tmp.write_text(json.dumps(manifest, indent=1))
        os.replace(tmp, d / "manifest.json")
    return d


def load_sharded(directory: str | Path, *, rank: int | None = None,
                 map_location: str | torch.device | None = "cpu") -> dict[str, Any]:
    """Returns {"step", "model", "optim" (this rank's shard or list of all), "manifest"}."""
    d = Path(directory)
    manifest = json.loads((d / "manifest.json").read_text())
    if manifest.get("format_version") != FORMAT_V2:
        raise ValueError("not a v2 sharded checkpoint")
    model = torch.load(d / manifest["model"], map_location=map_location, weights_only=False)
    if rank is None:
        optim = [torch.load(d / f, map_location=map_location, weights_only=False)
                 for f in manifest["optim"] if (d / f).exists()]
    else:
        f = d / manifest["optim"][rank]
        optim = torch.load(f, map_location=map_location, weights_only=False) if f.exists() else None
    return {"step": manifest["step"], "model": model, "optim": optim, "manifest": manifest}


def sharded_to_v1(directory: str | Path, out_path: str | Path) -> Path:
    """Gather a v2 checkpoint into a single v1 file (model + rank-0 optimizer state)."""
    data = load_sharded(directory)
    opt = data["optim"][0] if data["optim"] else None
    out = Path(out_path)
    _atomic_save({"format_version": FORMAT_V1, "step": data["step"], "model": data["model"],
                  "optimizer": opt, "extra": data["manifest"].get("extra")}, out)
    return out


# ------------------------------------------------------------------ expert layouts
_PER_EXPERT = re.compile(r"^(.*\.moe)\.routed_experts\.(\d+)\.(gate|up|down)_proj\.weight$")
_STACKED = re.compile(r"^(.*\.moe)\.grouped_experts\.(gate|up|down)_weight$")


def experts_to_stacked(state: dict[str, Tensor]) -> dict[str, Tensor]:
    out: dict[str, Tensor] = {}
    pending: dict[tuple[str, str], dict[int, Tensor]] = {}
    for k, v in state.items():
        m = _PER_EXPERT.match(k)
        if m:
            pending.setdefault((m.group(1), m.group(3)), {})[int(m.group(2))] = v
        else:
            out[k] = v
    for (prefix, kind), parts in pending.items():
        out[f"{prefix}.grouped_experts.{kind}_weight"] = torch.stack([parts[i] for i in sorted(parts)])
    return out


def experts_to_per_module(state: dict[str, Tensor]) -> dict[str, Tensor]:
    out: dict[str, Tensor] = {}
    for k, v in state.items():
        m = _STACKED.match(k)
        if m:
            for j in range(v.shape[0]):
                out[f"{m.group(1)}.routed_experts.{j}.{m.group(2)}_proj.weight"] = v[j].clone()
        else:
            out[k] = v
    return out


__all__ = [
    "experts_to_per_module",
    "experts_to_stacked",
    "load_checkpoint",
    "load_sharded",
    "save_checkpoint",
    "save_sharded",
    "sharded_to_v1",
]

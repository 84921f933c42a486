"""Weight initialisation schemes and u-muP parameter groups.

``normal`` (reference ``core/model.py:192-204``): N(0, initializer_range) for every
``nn.Linear`` / ``nn.Embedding`` instance except frozen weights and the mHC
``w_pre/w_res/w_post`` (kept at zero).  Quantised linears are not ``nn.Linear`` and
keep their kaiming init, as in the reference.

``umup`` (reference ``core/init.py:39-227``): embeddings N(0, 1); hidden linears
N(0, 1/sqrt(fan_in)); residual feeders (``output.final_proj``, ``down_proj``) get an
extra 1/sqrt(n_layers); mHC dynamic weights and frozen weights are skipped; tied
tensors are initialised once.  ``umup_param_groups`` returns an embedding group
(constant LR) and a hidden group (LR * base_width / width).
"""

from __future__ import annotations

import math

from torch import nn

RESIDUAL_FEEDER_SUFFIXES = ("output.final_proj.weight", "down_proj.weight")
MHC_DYNAMIC_NAMES = frozenset({"w_pre", "w_res", "w_post"})


def _is_mhc_dynamic(name: str) -> bool:
    return any(part in MHC_DYNAMIC_NAMES for part in name.split("."))


def normal_init(model: nn.Module, std: float) -> None:
    for name, mod in model.named_modules():
        if isinstance(mod, nn.Linear):
            if not mod.weight.requires_grad:
                continue
            if any(tag in name for tag in (".w_pre", ".w_res", ".w_post")):
                continue
            nn.init.normal_(mod.weight, mean=0.0, std=std)
        elif isinstance(mod, nn.Embedding):
            nn.init.normal_(mod.weight, mean=0.0, std=std)


def umup_init(model: nn.Module, *, n_layers: int, embedding_sigma: float = 1.0) -> None:
    if n_layers <= 0:
        raise ValueError(f"n_layers must be positive; got {n_layers}")
    done: set[int] = set()
    for _, mod in model.named_modules():
        if isinstance(mod, nn.Embedding) and mod.weight.requires_grad and id(mod.weight) not in done:
            nn.init.normal_(mod.weight, mean=0.0, std=embedding_sigma)
            done.add(id(mod.weight))
    for name, mod in model.named_modules():
        if not isinstance(mod, nn.Linear):
            continue
        wname = f"{name}.weight" if name else "weight"
        if _is_mhc_dynamic(wname) or not mod.weight.requires_grad or id(mod.weight) in done:
            continue
        std = 1.0 / math.sqrt(mod.in_features)
        if wname.endswith(RESIDUAL_FEEDER_SUFFIXES):
            std /= math.sqrt(n_layers)
        nn.init.normal_(mod.weight, mean=0.0, std=std)
        done.add(id(mod.weight))
        if mod.bias is not None and mod.bias.requires_grad:
            nn.init.zeros_(mod.bias)


def umup_param_groups(model: nn.Module, *, base_lr_hidden: float, base_lr_embedding: float,
                      base_width: int, actual_width: int | None = None) -> list[dict[str, object]]:
    if base_width <= 0:
        raise ValueError(f"base_width must be positive; got {base_width}")
    embed = getattr(model, "embed", None)
    if actual_width is None:
        if not isinstance(embed, nn.Embedding):
            raise ValueError("model has no `embed: nn.Embedding`; pass actual_width")
        actual_width = embed.embedding_dim
    if actual_width <= 0:
        raise ValueError(f"actual_width must be positive; got {actual_width}")
    embed_id = id(embed.weight) if isinstance(embed, nn.Embedding) else None
    seen: set[int] = set()
    emb, hid = [], []
    for _, p in model.named_parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        (emb if id(p) == embed_id else hid).append(p)
    return [
        {"name": "embedding", "params": emb, "lr": base_lr_embedding},
        {"name": "hidden", "params": hid, "lr": base_lr_hidden * base_width / actual_width},
    ]


def split_umup_groups(model: nn.Module, *, base_lr_hidden: float, base_lr_embedding: float,
                      base_width: int, actual_width: int | None = None
                      ) -> tuple[list[nn.Parameter], list[nn.Parameter], dict[str, float]]:
    g = {d["name"]: d for d in umup_param_groups(model, base_lr_hidden=base_lr_hidden,
                                                  base_lr_embedding=base_lr_embedding,
                                                  base_width=base_width, actual_width=actual_width)}
    return (list(g["embedding"]["params"]), list(g["hidden"]["params"]),  # type: ignore[call-overload]
            {"embedding": float(g["embedding"]["lr"]), "hidden": float(g["hidden"]["lr"])})  # type: ignore[arg-type]


__all__ = ["normal_init", "split_umup_groups", "umup_init", "umup_param_groups"]

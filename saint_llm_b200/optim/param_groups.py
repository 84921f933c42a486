"""Muon / AdamW parameter split (reference ``optim/param_groups.py:20-57``).

AdamW gets every parameter with fewer than 2 dims, the embedding / LM head, and
the mHC static biases and gating factors (``s_*``, ``alpha_*``); Muon gets every
other matrix (2-D, and here also the stacked 3-D expert weights).  Frozen
parameters go to neither.  Tied parameters are listed once.
"""

from __future__ import annotations

from torch import nn

ADAMW_NAME_PATTERNS: tuple[str, ...] = (
    "embed.weight", "lm_head.weight", ".s_pre", ".s_res", ".s_post",
    ".alpha_pre", ".alpha_res", ".alpha_post",
)


def split_for_muon_adamw(model: nn.Module) -> tuple[list[nn.Parameter], list[nn.Parameter]]:
    muon: list[nn.Parameter] = []
    adamw: list[nn.Parameter] = []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if p.dim() < 2 or any(pat in name for pat in ADAMW_NAME_PATTERNS):
            adamw.append(p)
        else:
            muon.append(p)
    return muon, adamw


__all__ = ["ADAMW_NAME_PATTERNS", "split_for_muon_adamw"]

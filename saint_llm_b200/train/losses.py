"""Training losses (reference ``training/losses.py:22-113``).

* ``cross_entropy_main``: shifted next-token CE on ``out["logits"]``.
* ``cross_entropy_with_mtp``: main + sum_k 0.3 * 0.9^k * CE(MTP head k, target shift
  k+2) (+ ``sequence_balance_weight * aux_loss``).
* ``make_loss_fn`` returns an ``nn.Module`` ``(model, batch) -> loss``.

``fused_lm_loss`` is the training path used on CUDA: the model returns hidden states
only and the LM-head GEMM, optional softcap, log-sum-exp and CE run chunk by chunk in
``ops.ce`` without materialising (B, T, V) logits -- identical value and gradients.
"""

from __future__ import annotations

import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.config import MoEConfig, MTPConfig


def cross_entropy_main(out: dict, batch: Tensor) -> Tensor:
    logits = out["logits"]
    if not isinstance(logits, Tensor):
        raise TypeError("out['logits'] must be a Tensor")
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), batch[:, 1:].reshape(-1))


def _add_aux(total: Tensor, out: dict, moe_cfg: MoEConfig | None) -> Tensor:
    if moe_cfg is None or moe_cfg.sequence_balance_weight == 0.0:
        return total
    aux = out.get("aux_loss") if isinstance(out, dict) else None
    if not isinstance(aux, Tensor):
        return total
    return total + moe_cfg.sequence_balance_weight * aux


def mtp_weight(cfg: MTPConfig, k: int) -> float:
    return cfg.loss_weight_main * (1.0 - cfg.loss_weight_decay) ** k


def cross_entropy_with_mtp(out: dict, batch: Tensor, *, cfg: MTPConfig,
                           moe_cfg: MoEConfig | None = None) -> Tensor:
    total = cross_entropy_main(out, batch)
    heads = out.get("mtp_logits") if isinstance(out, dict) else None
    if heads is not None and cfg.depth > 0:
        if not isinstance(heads, list):
            raise TypeError("out['mtp_logits'] must be a list of Tensors")
        for k, lg in enumerate(heads):
            shift = k + 2
            if batch.shape[1] <= shift:
                continue
            chunk = lg[:, :-shift].reshape(-1, lg.shape[-1])
            if chunk.shape[0] == 0:
                continue
            total = total + mtp_weight(cfg, k) * F.cross_entropy(chunk, batch[:, shift:].reshape(-1))
    return _add_aux(total, out, moe_cfg)


def fused_lm_loss(model: nn.Module, batch: Tensor, *, mtp_cfg: MTPConfig | None,
                  moe_cfg: MoEConfig | None) -> Tensor:
    """Same value as ``cross_entropy_with_mtp`` but never materialises the logits."""
    from saint_llm_b200.ops import ce

    out = model(batch, return_hidden_only=True)
    w = model.lm_head.weight
    cap = model.cfg.final_logit_softcap
    total = ce.lm_head_cross_entropy(out["hidden"][:, :-1], w, batch[:, 1:], softcap=cap)
    if mtp_cfg is not None and mtp_cfg.depth > 0:
        for k, mh in enumerate(out["mtp_hidden"]):
            shift = k + 2
            if batch.shape[1] <= shift:
                continue
            total = total + mtp_weight(mtp_cfg, k) * ce.lm_head_cross_entropy(
                mh[:, :-shift], w, batch[:, shift:], softcap=cap)
    return _add_aux(total, out, moe_cfg)


class _Loss(nn.Module):
    def __init__(self, mtp_cfg: MTPConfig | None, moe_cfg: MoEConfig | None, fused: bool | None) -> None:
        super().__init__()
        self.mtp_cfg = mtp_cfg
        self.moe_cfg = moe_cfg
        self.fused = fused

    def forward(self, model: nn.Module, batch: Tensor) -> Tensor:
        fused = self.fused
        if fused is None:
            from saint_llm_b200.ops import backend

            fused = backend.native_for(batch) and hasattr(model, "lm_head")
        if fused:
            return fused_lm_loss(model, batch, mtp_cfg=self.mtp_cfg, moe_cfg=self.moe_cfg)
        out = model(batch)
        if self.mtp_cfg is None:
            return _add_aux(cross_entropy_main(out, batch), out, self.moe_cfg)
        return cross_entropy_with_mtp(out, batch, cfg=self.mtp_cfg, moe_cfg=self.moe_cfg)


def make_loss_fn(mtp_cfg: MTPConfig | None = None, *, moe_cfg: MoEConfig | None = None,
                 fused: bool | None = None) -> nn.Module:
    """``fused=None`` picks the fused LM-head CE on CUDA and the logits path elsewhere."""
    return _Loss(mtp_cfg, moe_cfg, fused)


__all__ = ["cross_entropy_main", "cross_entropy_with_mtp", "fused_lm_loss", "make_loss_fn", "mtp_weight"]

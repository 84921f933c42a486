"""Muon (+ MuonClip QK-Clip) and a combined Muon/AdamW optimizer.

Muon per matrix W (n x m), reference ``optim/muon.py:57-192``::

    M <- mu M + G ;  U = mu M + G                    (Nesterov look-ahead)
    O = NS(U) * sqrt(max(n, m)) * gamma              (gamma = 0.18, RMS match to AdamW)
    W <- W (1 - lr wd) - lr O

Differences from the reference, each deliberate:

* 3-D stacked expert weights (E, out, in) are orthogonalised per expert slice (the
  reference raises; ``strict_2d=True`` restores that behaviour).
* All matrices of one shape are orthogonalised in one batched call (on CUDA: the
  native batched tensor-core GEMM, bf16 operands / fp32 accumulation).  On CPU the
  default NS is the reference's fp32 per-matrix iteration, so CPU results match.
* QK-Clip reads each attention layer's *device* max-logit buffer and rescales
  ``q_up`` / ``k_proj`` by ``sqrt(tau / max)`` where ``max > tau`` without a host
  sync; trigger counts are kept on the device and converted on access.

``MuonAdamW`` is one ``torch.optim.Optimizer`` whose param groups carry
``kind="muon"`` or ``kind="adamw"`` so a single object (and a single LR scheduler)
drives both halves of the V4 recipe.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable
from typing import Any, Protocol, runtime_checkable

import torch
from torch import Tensor, nn

from saint_llm_b200.optim.newton_schulz import STAGE1, STAGE2, batched_newton_schulz, hybrid_newton_schulz


def _grad(p: Tensor) -> Tensor | None:
    """fp32 ``main_grad`` when the training engine attached one, else ``.grad``."""
    mg = getattr(p, "main_grad", None)
    return mg if mg is not None else p.grad


def _active_grad(opt: torch.optim.Optimizer, p: Tensor) -> Tensor | None:
    """The gradient to step with, or None when the parameter is skipped this step (no gradient,
    or a ``param_filter`` -- e.g. ZeRO ownership -- excludes it)."""
    flt = getattr(opt, "param_filter", None)
    if flt is not None and not flt(p):
        return None
    return _grad(p)


@runtime_checkable
class _QKClippable(Protocol):
    _last_max_attn_logit: float

    def qk_clip_targets(self) -> list[Tensor]: ...


def _orthogonalize(updates: list[Tensor], group: dict[str, Any], impl: str) -> list[Tensor]:
    """NS-orthogonalise a list of same-shaped tensors (2-D or stacked 3-D)."""
    kw = dict(n_iter_stage1=group["ns_iter_stage1"], n_iter_stage2=group["ns_iter_stage2"],
              coeffs_stage1=tuple(group["ns_coeffs_stage1"]), coeffs_stage2=tuple(group["ns_coeffs_stage2"]))
    if impl == "reference":
        out = []
        for u in updates:
            out.append(hybrid_newton_schulz(u, **kw) if u.dim() == 2
                       else torch.stack([hybrid_newton_schulz(s, **kw) for s in u]))
        return out
    stacked = torch.cat([u.reshape(-1, *u.shape[-2:]) for u in updates])
    orth = batched_newton_schulz(stacked, precision="bf16" if impl == "batched_bf16" else "fp32", **kw)
    res, i = [], 0
    for u in updates:
        cnt = u.numel() // (u.shape[-2] * u.shape[-1])
        res.append(orth[i:i + cnt].reshape(u.shape))
        i += cnt
    return res


class _QKClipMixin:
    qk_clip_enabled: bool
    qk_clip_tau: float
    _qk_clip_layers: list[nn.Module]
    _qk_clip_counts: dict[int, Tensor]

    def _init_qk_clip(self, enabled: bool, tau: float, layers: Iterable[nn.Module] | None) -> None:
        if tau <= 0.0:
            raise ValueError(f"qk_clip_tau must be positive; got {tau}")
        self.qk_clip_enabled = enabled
        self.qk_clip_tau = tau
        self._qk_clip_layers = list(layers or [])
        self._qk_clip_counts = {}

    def register_qk_clip_layer(self, layer: nn.Module) -> None:
        if not isinstance(layer, _QKClippable):
            raise TypeError(f"Layer {type(layer).__name__} does not satisfy _QKClippable "
                            "protocol (needs _last_max_attn_logit and qk_clip_targets()).")
        self._qk_clip_layers.append(layer)

    @property
    def qk_clip_count(self) -> dict[int, int]:
        return {k: int(v) for k, v in self._qk_clip_counts.items() if int(v) > 0}

    @torch.no_grad()
    def _apply_qk_clip(self) -> None:
        tau = self.qk_clip_tau
        for layer in self._qk_clip_layers:
            buf = getattr(layer, "max_attn_logit", None)
            if isinstance(buf, Tensor):
                mx = buf.float()
                hit = mx > tau
                scale = torch.where(hit, torch.sqrt(tau / mx.clamp(min=1e-30)), torch.ones_like(mx))
                for w in layer.qk_clip_targets():
                    w.mul_(scale.to(w.dtype))
                cnt = self._qk_clip_counts.setdefault(id(layer), torch.zeros((), dtype=torch.long,
                                                                             device=mx.device))
                cnt.add_(hit.long())
            else:
                mxf = float(getattr(layer, "_last_max_attn_logit", 0.0))
                if mxf <= tau:
                    continue
                for w in layer.qk_clip_targets():
                    w.data.mul_((tau / mxf) ** 0.5)
                cnt = self._qk_clip_counts.setdefault(id(layer), torch.zeros((), dtype=torch.long))
                cnt.add_(1)


def _muon_defaults(lr: float, momentum: float, weight_decay: float, rms_rescale: float,
                   ns_iter_stage1: int, ns_iter_stage2: int, ns_coeffs_stage1: tuple[float, float, float],
                   ns_coeffs_stage2: tuple[float, float, float]) -> dict[str, Any]:
    if lr < 0.0:
        raise ValueError(f"Invalid lr {lr}")
    if not 0.0 <= momentum < 1.0:
        raise ValueError(f"Invalid momentum {momentum} (must be in [0, 1))")
    if weight_decay < 0.0:
        raise ValueError(f"Invalid weight_decay {weight_decay}")
    return dict(lr=lr, momentum=momentum, weight_decay=weight_decay, rms_rescale=rms_rescale,
                ns_iter_stage1=ns_iter_stage1, ns_iter_stage2=ns_iter_stage2,
                ns_coeffs_stage1=ns_coeffs_stage1, ns_coeffs_stage2=ns_coeffs_stage2)


@torch.no_grad()
def _tp_shard_step(opt: torch.optim.Optimizer, p: Tensor, g: Tensor, group: dict[str, Any], impl: str,
                   pg: Any, dim: int) -> None:
    """Muon step of a tensor-parallel shard of a matrix (rows ``dim=0`` or columns ``dim=1``
    split over the process group ``pg``): the momentum is element-wise, so it stays a shard,
    but Newton-Schulz orthogonalises the WHOLE matrix -- the shards' updates are gathered,
    orthogonalised identically on every rank, and each keeps its own slice."""
    import torch.distributed as dist

    lr, mu, wd, gamma = group["lr"], group["momentum"], group["weight_decay"], group["rms_rescale"]
    st = opt.state[p]
    if "momentum_buffer" not in st:
        st["momentum_buffer"] = torch.zeros_like(p)
    buf = st["momentum_buffer"]
    buf.mul_(mu).add_(g.to(buf.dtype))
    upd = (buf.float() * mu + g.float()).contiguous()
    ws, r = dist.get_world_size(pg), dist.get_rank(pg)
    parts = [torch.empty_like(upd) for _ in range(ws)]
    dist.all_gather(parts, upd, group=pg)
    full = torch.cat(parts, dim)
    o = _orthogonalize([full], group, "batched_bf16" if impl == "native" else impl)[0]
    n = p.shape[dim]
    local = o.narrow(dim, r * n, n)
    rows, cols = full.shape
    p.mul_(1.0 - lr * wd).add_((local * (math.sqrt(max(rows, cols)) * gamma)).to(p.dtype), alpha=-lr)


@torch.no_grad()
def _muon_group_step(opt: torch.optim.Optimizer, group: dict[str, Any], impl: str, strict_2d: bool,
                     chunk_elems: int = 1 << 28) -> None:
    lr, mu, wd, gamma = group["lr"], group["momentum"], group["weight_decay"], group["rms_rescale"]
    by_shape: dict[tuple[Any, ...], list[Tensor]] = {}
    shards = getattr(opt, "tp_shards", None) or {}
    for p in group["params"]:
        g = _active_grad(opt, p)
        if g is None:
            continue
        if id(p) in shards:
            _tp_shard_step(opt, p, g, group, impl, *shards[id(p)])
            continue
        if p.dim() != 2 and (strict_2d or p.dim() != 3):
            raise ValueError(f"Muon expects 2D matrix params; got shape {tuple(p.shape)}. "
                             "Use AdamW for 1D params (RMSNorm weights, biases, gating factors).")
        st = opt.state[p]
        if "momentum_buffer" not in st:
            st["momentum_buffer"] = torch.zeros_like(p)
        if impl != "native":
            st["momentum_buffer"].mul_(mu).add_(g.to(st["momentum_buffer"].dtype))
        by_shape.setdefault((*p.shape[-2:], str(p.device)), []).append(p)
    if impl == "native":
        for params in by_shape.values():
            _native_chunks(opt, params, group, chunk_elems)
        return
    for params in by_shape.values():
        # bounded working set: orthogonalise at most ~chunk_elems elements at a time
        chunk: list[Tensor] = []
        size = 0
        for i, p in enumerate(params):
            chunk.append(p)
            size += p.numel()
            if size >= chunk_elems or i == len(params) - 1:
                upd = [opt.state[q]["momentum_buffer"].float() * mu + _grad(q).float() for q in chunk]
                for q, o in zip(chunk, _orthogonalize(upd, group, impl), strict=True):
                    n, k = q.shape[-2:]
                    q.mul_(1.0 - lr * wd).add_((o * (math.sqrt(max(n, k)) * gamma)).to(q.dtype), alpha=-lr)
                chunk, size = [], 0


@torch.no_grad()
def _native_chunks(opt: torch.optim.Optimizer, params: list[Tensor], group: dict[str, Any], chunk_elems: int) -> None:
    """CUDA Muon for same-shaped matrices: fused momentum / normalise / apply kernels around
    the epilogue-fused batched Newton-Schulz (the momentum update happens here)."""
    from saint_llm_b200.ops import backend
    from saint_llm_b200.optim.newton_schulz import native_newton_schulz

    ext = backend.ext()
    lr, mu, wd, gamma = group["lr"], group["momentum"], group["weight_decay"], group["rms_rescale"]
    n, k = params[0].shape[-2:]
    slice_ = n * k
    i = 0
    while i < len(params):
        chunk, total = [], 0
        while i < len(params) and (not chunk or total + params[i].numel() <= chunk_elems):
            chunk.append(params[i])
            total += params[i].numel()
            i += 1
        y = torch.empty(total // slice_, n, k, dtype=torch.bfloat16, device=chunk[0].device)
        off = 0
        for q in chunk:
            cnt = q.numel() // slice_
            st = opt.state[q]
            g = _grad(q).float().contiguous()
            sumsq = torch.empty(cnt, dtype=torch.float32, device=q.device)
            ext.muon_momentum(st["momentum_buffer"], g, sumsq, slice_, float(mu))
            ext.muon_normalize(st["momentum_buffer"], g, sumsq, y[off:off + cnt], slice_, float(mu), 1.0e-7)
            off += cnt
        y = native_newton_schulz(y, group["ns_iter_stage1"], group["ns_iter_stage2"],
                                 tuple(group["ns_coeffs_stage1"]), tuple(group["ns_coeffs_stage2"]))
        off = 0
        scale = math.sqrt(max(n, k)) * gamma
        for q in chunk:
            cnt = q.numel() // slice_
            ext.muon_apply(q.data, y[off:off + cnt].contiguous(), 1.0 - lr * wd, lr * scale)
            off += cnt


def _resolve_impl(impl: str, params: Iterable[Tensor]) -> str:
    if impl != "auto":
        return impl
    for p in params:
        if p.is_cuda:
            from saint_llm_b200.ops import backend

            return "native" if backend.native_for(p) else "batched_bf16"
        return "reference"
    return "reference"


class Muon(_QKClipMixin, torch.optim.Optimizer):
    """Muon for matrix parameters (2-D, or stacked 3-D experts)."""

    def __init__(self, params: Iterable[nn.Parameter] | Iterable[dict[str, Any]], lr: float = 2.7e-4,
                 momentum: float = 0.95, weight_decay: float = 0.1, rms_rescale: float = 0.18,
                 ns_iter_stage1: int = 8, ns_iter_stage2: int = 2,
                 ns_coeffs_stage1: tuple[float, float, float] = STAGE1,
                 ns_coeffs_stage2: tuple[float, float, float] = STAGE2, *,
                 qk_clip_enabled: bool = True, qk_clip_tau: float = 100.0,
                 qk_clip_layers: Iterable[nn.Module] | None = None, ns_impl: str = "auto",
                 strict_2d: bool = False) -> None:
        super().__init__(params, _muon_defaults(lr, momentum, weight_decay, rms_rescale, ns_iter_stage1,
                                                ns_iter_stage2, ns_coeffs_stage1, ns_coeffs_stage2))
        self._init_qk_clip(qk_clip_enabled, qk_clip_tau, qk_clip_layers)
        self.ns_impl = ns_impl
        self.param_filter: Callable[[Tensor], bool] | None = None
        self.strict_2d = strict_2d

    @torch.no_grad()
    def step(self, closure: Callable[[], Tensor] | None = None) -> Tensor | None:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            _muon_group_step(self, group, _resolve_impl(self.ns_impl, group["params"]), self.strict_2d)
        if self.qk_clip_enabled and self._qk_clip_layers:
            self._apply_qk_clip()
        return loss


class MuonAdamW(_QKClipMixin, torch.optim.Optimizer):
    """One optimizer for the V4 split: groups with ``kind="muon"`` or ``kind="adamw"``."""

    def __init__(self, muon_params: Iterable[nn.Parameter], adamw_params: Iterable[nn.Parameter], *,
                 lr: float = 2.7e-4, momentum: float = 0.95, weight_decay: float = 0.1,
                 rms_rescale: float = 0.18, adamw_lr: float | None = None,
                 betas: tuple[float, float] = (0.9, 0.95), eps: float = 1e-20,
                 adamw_weight_decay: float | None = None, qk_clip_enabled: bool = True,
                 qk_clip_tau: float = 100.0, qk_clip_layers: Iterable[nn.Module] | None = None,
                 ns_impl: str = "auto") -> None:
        muon_defaults = _muon_defaults(lr, momentum, weight_decay, rms_rescale, 8, 2, STAGE1, STAGE2)
        groups = [
            {"params": list(muon_params), "kind": "muon", **muon_defaults},
            {"params": list(adamw_params), "kind": "adamw", "lr": adamw_lr if adamw_lr is not None else lr,
             "betas": betas, "eps": eps,
             "weight_decay": adamw_weight_decay if adamw_weight_decay is not None else weight_decay},
        ]
        super().__init__([g for g in groups if g["params"]], {})
        self._init_qk_clip(qk_clip_enabled, qk_clip_tau, qk_clip_layers)
        self.ns_impl = ns_impl
        self.param_filter: Callable[[Tensor], bool] | None = None

    @torch.no_grad()
    def step(self, closure: Callable[[], Tensor] | None = None) -> Tensor | None:
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            if group["kind"] == "muon":
                _muon_group_step(self, group, _resolve_impl(self.ns_impl, group["params"]), False)
            else:
                self._adamw_group_step(group)
        if self.qk_clip_enabled and self._qk_clip_layers:
            self._apply_qk_clip()
        from saint_llm_b200.ops.fp8 import bump_weight_epoch

        bump_weight_epoch()  # cached FP8 weight copies are stale now
        return loss

    @torch.no_grad()
    def init_state(self) -> int:
        """Allocate every state buffer the first ``step`` would create (Muon momentum, AdamW
        moments) now, for the parameters this rank updates (``param_filter``), so memory
        planning done before the first step -- a CUDA-graph capture -- sees them.  Returns
        the bytes allocated."""
        flt = self.param_filter
        n = 0
        for group in self.param_groups:
            for p in group["params"]:
                if not p.requires_grad or (flt is not None and not flt(p)):
                    continue
                st = self.state[p]
                if group["kind"] == "muon":
                    if "momentum_buffer" not in st:
                        st["momentum_buffer"] = torch.zeros_like(p)
                        n += p.numel() * p.element_size()
                elif not st:
                    st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                    st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                    st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
                    n += 8 * p.numel()
        return n

    @torch.no_grad()
    def _adamw_group_step(self, group: dict[str, Any]) -> None:
        params = [p for p in group["params"] if _active_grad(self, p) is not None]
        if not params:
            return
        b1, b2 = group["betas"]
        lr, eps, wd = group["lr"], group["eps"], group["weight_decay"]
        for p in params:
            st = self.state[p]
            if not st:
                st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
        if params[0].is_cuda:
            from saint_llm_b200.ops import backend

            if backend.native_for(params[0]):
                from saint_llm_b200.ops import optim_kernels

                optim_kernels.adamw_step(params, [self.state[p] for p in params], lr=lr, beta1=b1,
                                         beta2=b2, eps=eps, weight_decay=wd)
                return
        for p in params:
            st = self.state[p]
            st["step"] += 1
            t = float(st["step"])
            g = _grad(p).float()
            st["exp_avg"].mul_(b1).add_(g, alpha=1 - b1)
            st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = (st["exp_avg_sq"] / (1 - b2 ** t)).sqrt_().add_(eps)
            upd = st["exp_avg"] / (1 - b1 ** t) / denom
            p.mul_(1 - lr * wd).add_(upd.to(p.dtype), alpha=-lr)


__all__ = ["Muon", "MuonAdamW"]

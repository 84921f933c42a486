"""Expert parallelism (EP).

Experts are partitioned contiguously: rank r of the EP group owns experts
``[r*E/N, (r+1)*E/N)``.

Reference-compatible API (``distributed/expert_parallel.py:47-276``):
``dispatch_tokens_by_expert(tokens, expert_ids, n_experts=..., world_size=None,
group=None) -> DispatchPlan`` (stable sort by destination rank, counts all-to-all,
payload all-to-all; a ``world_size`` different from the process group's runs the same
permutation without communication -- "simulation mode") and
``combine_outputs_by_expert(expert_out, plan)`` (reverse all-to-all + un-permute).

Training path (``moe_forward_ep``): router -> one row per (token, slot) sorted by
destination rank -> autograd all-to-all -> the rank's local experts on the tensor
cores (the grouped GEMMs of ``ops.moe_native`` with k = 1) -> reverse all-to-all ->
gate-weighted sum per token.  The all-to-all here is NCCL (gloo on CPU); gradients
flow through ``torch.distributed.nn`` all-to-alls.

``setup_expert_parallel(model)`` shards every grouped expert pool to the local slice,
marks the layers and returns the gradient synchroniser: replicated (non-expert)
gradients are averaged across ranks (bucketed all-reduce); expert gradients, already
complete on their owner, are divided by the world size so both follow the same
global-mean loss.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor, nn


@dataclass(frozen=True)
class DispatchPlan:
    permuted_tokens: Tensor
    send_counts: Tensor
    recv_counts: Tensor
    sort_indices: Tensor
    local_expert_offsets: Tensor
    n_local_tokens: int
    world_size: int = 1
    simulated: bool = True


def _pg_size(group: dist.ProcessGroup | None) -> int:
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def dispatch_tokens_by_expert(tokens: Tensor, expert_ids: Tensor, *, n_experts: int, world_size: int | None = None,
                              group: dist.ProcessGroup | None = None) -> DispatchPlan:
    if tokens.dim() != 2:
        raise ValueError(f"tokens must be (N, D); got shape {tuple(tokens.shape)}")
    if expert_ids.shape[0] != tokens.shape[0]:
        raise ValueError(f"expert_ids length {expert_ids.shape[0]} != tokens batch {tokens.shape[0]}")
    if n_experts <= 0:
        raise ValueError(f"n_experts must be positive; got {n_experts}")
    pg_ws = _pg_size(group)
    ws = world_size if world_size is not None else pg_ws
    if n_experts % ws:
        raise ValueError(f"n_experts {n_experts} must be divisible by world_size {ws}")
    real = ws == pg_ws and pg_ws > 1
    per = n_experts // ws
    dest = (expert_ids // per).clamp(0, ws - 1)
    order = torch.argsort(dest, stable=True)
    send = tokens.index_select(0, order)
    send_counts = torch.bincount(dest, minlength=ws).to(torch.int64)
    # per-local-expert offsets of the rows this rank receives (its own slice when simulated)
    if real:
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=group)
        rs, ss = recv_counts.tolist(), send_counts.tolist()
        recv = tokens.new_empty(sum(rs), tokens.shape[1])
        dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=rs, input_split_sizes=ss, group=group)
    else:
        recv_counts, recv = send_counts.clone(), send
    offsets = torch.zeros(per, dtype=torch.int64, device=tokens.device)
    return DispatchPlan(recv, send_counts, recv_counts, order, offsets, tokens.shape[0], ws, not real)


def combine_outputs_by_expert(expert_out: Tensor, plan: DispatchPlan, *,
                              group: dist.ProcessGroup | None = None) -> Tensor:
    if expert_out.shape[0] != plan.permuted_tokens.shape[0]:
        raise ValueError("expert_out rows must match the dispatched rows")
    if not plan.simulated:
        back = expert_out.new_empty(plan.n_local_tokens, *expert_out.shape[1:])
        dist.all_to_all_single(back, expert_out.contiguous(), output_split_sizes=plan.send_counts.tolist(),
                               input_split_sizes=plan.recv_counts.tolist(), group=group)
    else:
        back = expert_out
    out = torch.empty_like(back)
    out.index_copy_(0, plan.sort_indices, back)
    return out


# ------------------------------------------------------------------ training path
def _a2a(x: Tensor, out_splits: list[int], in_splits: list[int], group: dist.ProcessGroup | None) -> Tensor:
    from torch.distributed.nn.functional import all_to_all_single

    out = x.new_empty(sum(out_splits), *x.shape[1:])
    return all_to_all_single(out, x.contiguous(), output_split_sizes=out_splits, input_split_sizes=in_splits,
                             group=group)


def moe_forward_ep(layer: nn.Module, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
    """``DeepSeekMoE`` forward with the routed experts sharded over the EP group."""
    from saint_llm_b200.ops import backend

    if getattr(layer, "ep_comm", None) is not None and backend.native_for(x):
        from saint_llm_b200.parallel.ep_p2p import moe_forward_p2p

        return moe_forward_p2p(layer, x, token_ids, is_visual)

    b, t, d = x.shape
    h = layer.norm(x)
    idx, gate, aux = layer.route(h, token_ids, is_visual)
    layer._last_aux_loss = aux
    k = layer.cfg.experts_per_token
    T = b * t
    h2 = h.reshape(T, d)
    group = layer.ep_group
    ws, rank = layer.ep_size, layer.ep_rank
    e_loc = layer.cfg.routed_experts // ws
    flat_e = idx.reshape(-1)
    dest = flat_e // e_loc
    order = torch.argsort(dest, stable=True)
    send_counts = torch.bincount(dest, minlength=ws).to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    ss, rs = send_counts.tolist(), recv_counts.tolist()
    send_x = h2.index_select(0, order // k)
    send_e = flat_e.index_select(0, order).contiguous()
    recv_x = _a2a(send_x, rs, ss, group)
    recv_e = send_e.new_empty(sum(rs))
    dist.all_to_all_single(recv_e, send_e, output_split_sizes=rs, input_split_sizes=ss, group=group)
    local_ids = (recv_e - rank * e_loc).view(-1, 1)
    ge = layer.grouped_experts
    native = backend.native_for(x)
    if native:
        from saint_llm_b200.ops.moe_native import routed_experts, shared_experts

        ones = torch.ones(local_ids.shape[0], 1, dtype=torch.float32, device=x.device)
        y_recv = routed_experts(recv_x, local_ids, ones, ge)
    else:
        ones = torch.ones(local_ids.shape[0], 1, dtype=torch.float32, device=x.device)
        y_recv = ge(recv_x, local_ids, ones)
    back = _a2a(y_recv, ss, rs, group)
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel(), device=order.device)
    y_pair = back.index_select(0, inv).view(T, k, d)
    out = (y_pair.float() * gate.reshape(T, k, 1).float()).sum(1).to(h2.dtype)
    if native:
        sh = shared_experts(h2, layer.shared_experts)
        if sh is not None:
            out = out + sh
    else:
        for expert in layer.shared_experts:
            out = out + expert(h2)
    return out.view(b, t, d)


def shard_grouped_experts(model: nn.Module, rank: int, ws: int, group: dist.ProcessGroup | None) -> list[Tensor]:
    """Keep only this rank's expert slice; returns the sharded (expert) parameters."""
    from saint_llm_b200.models.moe import DeepSeekMoE

    expert_params: list[Tensor] = []
    for mod in model.modules():
        if not isinstance(mod, DeepSeekMoE):
            continue
        ge = mod.grouped_experts
        if ge is None:
            raise ValueError("expert parallelism needs the stacked (moe_use_grouped_gemm) expert layout")
        E = ge.n_experts
        if E % ws:
            raise ValueError(f"routed_experts {E} not divisible by EP size {ws}")
        per = E // ws
        for name in ("gate_weight", "up_weight", "down_weight"):
            full = getattr(ge, name)
            local = nn.Parameter(full.data[rank * per:(rank + 1) * per].clone(), requires_grad=full.requires_grad)
            setattr(ge, name, local)
            expert_params.append(local)
        ge.n_global_experts = E
        ge.n_experts = per
        mod.ep_group = group
        mod.ep_size = ws
        mod.ep_rank = rank
    return expert_params


def make_grad_sync(expert_params: list[Tensor], group: dist.ProcessGroup | None,
                   bucket_bytes: int = 256 << 20, *, exclude: set[int] | None = None,
                   expert_div: int | None = None) -> Callable[[list[Tensor]], None]:
    """Average replicated main_grads across ranks (bucketed all-reduce); scale expert grads by
    1/``expert_div`` (default: the group size).  Parameters whose ids are in ``exclude`` are
    left alone (another group reduces them)."""
    ws = dist.get_world_size(group)
    eids = {id(p) for p in expert_params}
    skip = eids | (exclude or set())
    ediv = expert_div or ws

    def sync(params: list[Tensor]) -> None:
        rep = [p.main_grad for p in params if id(p) not in skip]  # type: ignore[attr-defined]
        bucket: list[Tensor] = []
        size = 0
        for i, g in enumerate(rep):
            bucket.append(g)
            size += g.numel() * 4
            if size >= bucket_bytes or i == len(rep) - 1:
                flat = torch.cat([x.reshape(-1) for x in bucket])
                dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
                flat.div_(ws)
                off = 0
                for x in bucket:
                    x.copy_(flat[off:off + x.numel()].view_as(x))
                    off += x.numel()
                bucket, size = [], 0
        for p in params:
            if id(p) in eids:
                p.main_grad.div_(ediv)  # type: ignore[attr-defined]

    return sync


def _mean_over(grads: list[Tensor], group: dist.ProcessGroup | None, bucket_bytes: int = 256 << 20) -> None:
    """In-place mean of ``grads`` over ``group`` (bucketed fp32 all-reduces)."""
    ws = dist.get_world_size(group)
    i = 0
    while i < len(grads):
        bucket, size = [], 0
        while i < len(grads) and (not bucket or size < bucket_bytes):
            bucket.append(grads[i])
            size += grads[i].numel() * 4
            i += 1
        flat = torch.cat([x.reshape(-1).float() for x in bucket])
        dist.all_reduce(flat, group=group)
        flat.div_(ws)
        off = 0
        for x in bucket:
            x.copy_(flat[off:off + x.numel()].view_as(x))
            off += x.numel()


def _sync_attention_logits(model: nn.Module, group: dist.ProcessGroup | None) -> None:
    """Global (MAX over ranks) attention-logit telemetry, so MuonClip makes the same
    decision for the replicated ``q_up`` / ``k_proj`` on every rank."""
    bufs = [m.max_attn_logit for m in model.modules() if isinstance(getattr(m, "max_attn_logit", None), Tensor)]
    if bufs:
        flat = torch.stack([b.float() for b in bufs])
        dist.all_reduce(flat, op=dist.ReduceOp.MAX, group=group)
        for b, v in zip(bufs, flat, strict=True):
            b.copy_(v)


class ParallelSync:
    """Gradient synchroniser returned by ``setup_expert_parallel`` (callable as
    ``sync(params)`` after the backward); ``post_step()`` runs after the optimizer.

    Plain mode: replicated gradients are all-reduced and every rank updates every
    replicated parameter.  ZeRO mode (hybrid ZeRO, reference planner
    ``distributed/zero.py:47-216`` with a runtime): each replicated parameter has one
    owner chosen by the LPT planner over Muon / AdamW costs; gradients are reduced to the
    owner only, only the owner runs the optimizer on it (``optimizer.param_filter``), and
    the updated parameters are broadcast from their owners.  Expert parameters are local
    to their rank in both modes (their gradients are divided by the world size so the
    loss is the global mean).

    With tensor parallelism composed in (``parallel.tp_ep``), three more sets: ``dp_params``
    (head-sharded attention weights: each TP rank holds a different slice) are averaged over
    ``dp_group`` (the ranks holding the same slice) and updated on every rank, outside ZeRO;
    ``partial_params`` (gradients that are partial sums over the TP ranks of one replica:
    replicated attention weights, MoE router / norm / shared experts) are scaled by
    ``partial_scale`` after the group mean; the expert gradients are divided by
    ``expert_div`` (the number of data replicas) instead of the group size."""

    def __init__(self, model: nn.Module, expert_params: list[Tensor], group: dist.ProcessGroup | None,
                 *, zero: bool, overlap_reduce: bool = False, zero_transport: str = "nccl",
                 timeout_s: float = 30.0, dp_params: list[Tensor] | None = None,
                 dp_group: dist.ProcessGroup | None = None, partial_params: list[Tensor] | None = None,
                 partial_scale: float = 1.0, expert_div: int | None = None) -> None:
        self.model, self.group = model, group
        self.ws = dist.get_world_size(group)
        self.expert_ids = {id(p) for p in expert_params}
        self.expert_params = expert_params
        self.expert_div = expert_div or self.ws
        self.dp_params = list(dp_params or [])
        self.dp_ids = {id(p) for p in self.dp_params}
        self.dp_group = dp_group
        self.partial_params = list(partial_params or [])
        self.partial_scale = partial_scale
        self.tp_shards: dict[int, tuple[object, int]] = {}
        self.zero = None
        self._plain = None
        self.overlap = False
        if zero:
            from saint_llm_b200.optim import split_for_muon_adamw
            from saint_llm_b200.parallel.zero import ZeroOptimizerSync

            muon, adamw = split_for_muon_adamw(model)
            kinds = {id(p): "muon" for p in muon} | {id(p): "adamw" for p in adamw}
            rep = [p for p in model.parameters()
                   if id(p) not in self.expert_ids and id(p) not in self.dp_ids and p.requires_grad]
            rep_kinds = [kinds.get(id(p), "adamw") for p in rep]
            if zero_transport == "auto":
                zero_transport = "p2p" if rep and rep[0].is_cuda else "nccl"
            if zero_transport == "p2p":
                from saint_llm_b200.parallel.zero_p2p import PeerZeroSync

                self.zero = PeerZeroSync(rep, rep_kinds, group=group, timeout_s=timeout_s)
            elif zero_transport == "nccl":
                self.zero = ZeroOptimizerSync(rep, rep_kinds, group=group)
            else:
                raise ValueError(f"unknown ZeRO transport {zero_transport!r}")
            blocks = list(getattr(model, "blocks", []))
            if overlap_reduce and blocks:
                self._hook_blocks(blocks)
        else:
            self._plain = make_grad_sync(expert_params, group, exclude=self.dp_ids, expert_div=self.expert_div)

    def _hook_blocks(self, blocks: list[nn.Module]) -> None:
        """Overlapped reduce: block i's backward hook reduces block i + 1's group (one
        block of slack, so late gradient accumulations of block i + 1 have landed)."""
        self.zero.overlap_groups([[p for p in b.parameters() if p.requires_grad] for b in blocks])
        n = len(blocks)
        for i, b in enumerate(blocks):
            if i + 1 < n:
                b.register_full_backward_hook(lambda m, gi, go, g=i + 1: self.zero.group_done(g))
        self.overlap = True

    def before_last_backward(self) -> None:
        """Called by ``TrainStep`` before the backward of a step's last micro-batch."""
        if self.overlap:
            self.zero.final_micro = True

    def is_updated_here(self, p: Tensor) -> bool:
        return self.zero is None or id(p) in self.expert_ids or id(p) in self.dp_ids or self.zero.is_owned(p)

    def configure_optimizer(self, optimizer: torch.optim.Optimizer) -> None:
        if self.zero is not None:
            optimizer.param_filter = self.is_updated_here  # type: ignore[attr-defined]
        if self.tp_shards:
            optimizer.tp_shards = self.tp_shards  # type: ignore[attr-defined]

    @staticmethod
    def _grad(p: Tensor) -> Tensor:
        g = getattr(p, "main_grad", None)
        return g if g is not None else p.grad

    @torch.no_grad()
    def __call__(self, params: list[Tensor]) -> None:
        _sync_attention_logits(self.model, self.group)
        if self._plain is not None:
            self._plain(params)
        else:
            if self.overlap:
                self.zero.finish_reduce()
            else:
                self.zero.reduce_grads()
            for p in self.expert_params:
                self._grad(p).div_(self.expert_div)
        if self.partial_scale != 1.0:
            for p in self.partial_params:
                g = self._grad(p)
                if g is not None:
                    g.mul_(self.partial_scale)
        if self.dp_params:
            _mean_over([g for p in self.dp_params if (g := self._grad(p)) is not None], self.dp_group)

    @torch.no_grad()
    def post_step(self) -> None:
        if self.zero is not None:
            self.zero.broadcast_params()
            from saint_llm_b200.ops.fp8 import bump_weight_epoch

            bump_weight_epoch()  # broadcast weights replace the local ones


def setup_expert_parallel(model: nn.Module, group: dist.ProcessGroup | None = None, *, transport: str = "auto",
                          capacity_factor: float | None = None, zero: bool = False, timeout_s: float = 30.0,
                          overlap_reduce: bool = False, zero_transport: str = "nccl",
                          **tp_sets: object) -> ParallelSync:
    """Shard the experts over ``group`` and return the gradient synchroniser.

    ``transport``: "p2p" moves tokens with the peer-memory kernels of ``parallel.ep_p2p``
    (CUDA only), "nccl" with ``all_to_all_single``; "auto" picks p2p on CUDA.
    ``zero``: hybrid ZeRO for the replicated parameters (see ``ParallelSync``); call
    ``sync.configure_optimizer(opt)`` once and ``sync.post_step()`` after every step.
    ``overlap_reduce`` (with ``zero``): issue each block's owner reductions from its
    backward hook during the last micro-batch.  ``zero_transport`` (with ``zero``): "nccl"
    reduce / broadcast, "p2p" (``parallel.zero_p2p``: owners pull over NVLink peer memory),
    or "auto" (p2p for CUDA parameters).  ``timeout_s``: bound of every cross-GPU flag wait of the peer-memory kernels.
    ``tp_sets``: the tensor-parallel parameter sets of ``ParallelSync`` (``dp_params``, ``dp_group``,
    ``partial_params``, ``partial_scale``, ``expert_div``), given by ``parallel.tp_ep``."""
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    sync = ParallelSync(model, shard_grouped_experts(model, rank, ws, group), group, zero=zero,
                        overlap_reduce=overlap_reduce, zero_transport=zero_transport, timeout_s=timeout_s,
                        **tp_sets)  # type: ignore[arg-type]
    dev = next(model.parameters()).device
    if transport not in ("auto", "p2p", "nccl"):
        raise ValueError(f"unknown transport {transport!r}")
    if transport == "p2p" or (transport == "auto" and dev.type == "cuda"):
        if dev.type != "cuda":
            raise ValueError("the p2p transport needs CUDA parameters")
        from saint_llm_b200.parallel.ep_p2p import attach_p2p_comm

        attach_p2p_comm(model, group, dev, capacity_factor=capacity_factor, timeout_s=timeout_s)
    return sync


__all__ = [
    "DispatchPlan",
    "ParallelSync",
    "combine_outputs_by_expert",
    "dispatch_tokens_by_expert",
    "make_grad_sync",
    "moe_forward_ep",
    "setup_expert_parallel",
    "shard_grouped_experts",
]

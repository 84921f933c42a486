"""Tensor parallelism for the attention blocks (absent in the reference, whose only
multi-GPU training path is FSDP2; the build plan asks for TP=2 on attention).

Heads are sharded: rank r of a TP group of size t keeps heads ``[r*H/t, (r+1)*H/t)``:
the matching rows of ``q_up``, the matching entries of the sink logits, and whole
groups of the grouped output projection (``g/t`` group linears) with the matching
column slice of ``final_proj``.  Everything else inside the attention module (the
query compressor, the single MQA K/V head, norms, the compressors, the lightning
indexer) is replicated and computed identically on every rank.

Collectives (Megatron-style, differentiable):

* the module input goes through ``copy_to_tp`` (identity forward, all-reduce of the
  input gradient backward): every path from ``h`` inside the module only sees local
  heads, so the full ``dh`` is the sum over ranks;
* the output of the row-sharded ``final_proj`` goes through ``reduce_from_tp``
  (all-reduce forward, identity backward);
* gradients of the replicated parameters are partial sums over the local heads, so
  ``TPGradSync`` all-reduces them after the backward.

``all_gather_seq`` / ``reduce_scatter_seq`` are the sequence-parallel pair (gather
before a column-parallel GEMM, reduce-scatter after a row-parallel one).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor, nn


def _ws(group: dist.ProcessGroup | None) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, group: Any) -> Tensor:  # type: ignore[override]
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, group: Any) -> Tensor:  # type: ignore[override]
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return g, None


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, group: Any, dim: int) -> Tensor:  # type: ignore[override]
        ctx.group, ctx.dim = group, dim
        parts = [torch.empty_like(x) for _ in range(_ws(group))]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=dim)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return _scatter_sum(g, ctx.group, ctx.dim), None, None


def _scatter_sum(x: Tensor, group: Any, dim: int) -> Tensor:
    parts = [p.contiguous() for p in x.chunk(_ws(group), dim=dim)]
    out = torch.empty_like(parts[0])
    dist.reduce_scatter(out, parts, group=group)
    return out


class _ScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, group: Any, dim: int) -> Tensor:  # type: ignore[override]
        ctx.group, ctx.dim = group, dim
        return _scatter_sum(x, group, dim)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        return _GatherSeq.apply(g, ctx.group, ctx.dim), None, None


class _SplitBatch(torch.autograd.Function):
    """This rank's 1/ws of dim 0 of a tensor that is identical on the group's ranks; the
    backward gathers the shares' gradients, so every rank again holds the full gradient."""

    @staticmethod
    def forward(ctx, x: Tensor, group: Any) -> Tensor:  # type: ignore[override]
        ctx.group = group
        ws, r = _ws(group), dist.get_rank(group)
        n = x.shape[0] // ws
        return x[r * n:(r + 1) * n].contiguous()

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        parts = [torch.empty_like(g) for _ in range(_ws(ctx.group))]
        dist.all_gather(parts, g.contiguous(), group=ctx.group)
        return torch.cat(parts, 0), None


class _GatherBatch(torch.autograd.Function):
    """Concatenate the ranks' shares along dim 0; the gradient arriving is identical on every
    rank (replicated computation downstream), so each rank keeps its own share of it."""

    @staticmethod
    def forward(ctx, x: Tensor, group: Any) -> Tensor:  # type: ignore[override]
        ctx.group, ctx.n = group, x.shape[0]
        parts = [torch.empty_like(x) for _ in range(_ws(group))]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, 0)

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        r = dist.get_rank(ctx.group)
        return g[r * ctx.n:(r + 1) * ctx.n].contiguous(), None


def split_batch_tp(x: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    return _SplitBatch.apply(x, group)


def gather_batch_tp(x: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    return _GatherBatch.apply(x, group)


def copy_to_tp(x: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x: Tensor, group: dist.ProcessGroup | None = None) -> Tensor:
    return _ReduceFromTP.apply(x, group)


def all_gather_seq(x: Tensor, group: dist.ProcessGroup | None = None, dim: int = 1) -> Tensor:
    return _GatherSeq.apply(x, group, dim)


def reduce_scatter_seq(x: Tensor, group: dist.ProcessGroup | None = None, dim: int = 1) -> Tensor:
    return _ScatterSeq.apply(x, group, dim)


class ColumnParallelLinear(nn.Module):
    """``y[..., local out slice] = x W_local^T``; the input gradient is all-reduced."""

    def __init__(self, full: nn.Module, rank: int, ws: int, group: dist.ProcessGroup | None) -> None:
        super().__init__()
        out = full.weight.shape[0]
        if out % ws:
            raise ValueError(f"out_features {out} not divisible by TP size {ws}")
        n = out // ws
        self.weight = nn.Parameter(full.weight.data[rank * n:(rank + 1) * n].clone())
        self.group = group

    def forward(self, x: Tensor) -> Tensor:
        return torch.nn.functional.linear(copy_to_tp(x, self.group), self.weight)


class RowParallelLinear(nn.Module):
    """``y = sum_ranks x_local W[:, local in slice]^T``; all-reduce of the output."""

    def __init__(self, full: nn.Module, rank: int, ws: int, group: dist.ProcessGroup | None,
                 *, reduce: bool = True) -> None:
        super().__init__()
        inp = full.weight.shape[1]
        if inp % ws:
            raise ValueError(f"in_features {inp} not divisible by TP size {ws}")
        n = inp // ws
        self.weight = nn.Parameter(full.weight.data[:, rank * n:(rank + 1) * n].clone())
        self.group, self.reduce = group, reduce

    def forward(self, x: Tensor) -> Tensor:
        y = torch.nn.functional.linear(x, self.weight)
        return reduce_from_tp(y, self.group) if self.reduce else y


def _tp_pre_hook(group: dist.ProcessGroup | None):
    def hook(module: nn.Module, args: tuple, kwargs: dict) -> tuple[tuple, dict]:
        return (copy_to_tp(args[0], group), *args[1:]), kwargs

    return hook


def _tp_post_hook(group: dist.ProcessGroup | None):
    def hook(module: nn.Module, args: tuple, kwargs: dict, out: Tensor) -> Tensor:
        return reduce_from_tp(out, group)

    return hook


def shard_attention_heads(attn: nn.Module, group: dist.ProcessGroup | None = None, comm: Any = None) -> list[Tensor]:
    """Shard one SWA/CSA/HCA/NSA module's heads over ``group`` in place (the module keeps
    its class; the input copy and output all-reduce are forward hooks); returns the
    replicated parameters whose gradients need ``TPGradSync``.

    ``comm`` (a ``tp_p2p.PeerTPComm``): the NVLink peer-memory transport.  The output
    projection then runs as one GEMM that pushes its tiles to the peer while it computes
    (``PeerRowParallelLinear``), the input gradient is reduced by the peer kernels, and no
    NCCL call is made for the block's activations."""
    rank, ws = dist.get_rank(group), _ws(group)
    cfg = attn.attn_cfg
    H, g = cfg.query_heads, cfg.output_proj_groups
    if H % ws or g % ws:
        raise ValueError(f"query_heads {H} and output_proj_groups {g} must be divisible by TP size {ws}")
    hd = cfg.head_dim
    attn.attn_cfg = cfg.model_copy(update={"query_heads": H // ws, "output_proj_groups": g // ws})
    sharded: set[int] = set()
    rows = slice(rank * (H // ws) * hd, (rank + 1) * (H // ws) * hd)
    attn.q_up.weight = nn.Parameter(attn.q_up.weight.data[rows].clone())
    attn.q_up.out_features = attn.q_up.weight.shape[0]
    sharded.add(id(attn.q_up.weight))
    if attn.sink_logit is not None:
        attn.sink_logit = nn.Parameter(attn.sink_logit.data[rank * (H // ws):(rank + 1) * (H // ws)].clone())
        sharded.add(id(attn.sink_logit))
    out = attn.output
    per = g // ws
    out.group_projs = nn.ModuleList(list(out.group_projs)[rank * per:(rank + 1) * per])
    out.n_groups = per
    for p in out.group_projs.parameters():
        sharded.add(id(p))
    fp = out.final_proj
    cols = slice(rank * per * out.d_g, (rank + 1) * per * out.d_g)
    fp.weight = nn.Parameter(fp.weight.data[:, cols].clone())
    fp.in_features = fp.weight.shape[1]
    sharded.add(id(fp.weight))
    if comm is not None:
        from saint_llm_b200.parallel.tp_p2p import PeerRowParallelLinear, peer_copy_to_tp

        out.final_proj = PeerRowParallelLinear(fp.weight, comm)
        attn.register_forward_pre_hook(
            lambda m, args, kwargs: ((peer_copy_to_tp(args[0], comm), *args[1:]), kwargs), with_kwargs=True)
    else:
        attn.register_forward_pre_hook(_tp_pre_hook(group), with_kwargs=True)
        attn.register_forward_hook(_tp_post_hook(group), with_kwargs=True)
    attn.tp_group = group
    return [p for p in attn.parameters() if id(p) not in sharded and p.requires_grad]


def split_moe_batches(model: nn.Module, group: dist.ProcessGroup | None = None) -> list[nn.Module]:
    """Make every MoE layer route only this TP rank's share of the batch (the TP ranks hold
    the same sequences after the head-sharded attention) and gather the outputs, so the
    routed experts see each token once per TP group.  Returns the MoE layers; the gradients
    of their non-expert parameters are then partial sums over the TP ranks."""
    from saint_llm_b200.models.moe import DeepSeekMoE

    ws, rank = _ws(group), dist.get_rank(group)
    layers = [m for m in model.modules() if isinstance(m, DeepSeekMoE)]
    for m in layers:
        m.tp_group, m.tp_size, m.tp_rank = group, ws, rank
    return layers


class TPGradSync:
    """Sum the gradients (``main_grad`` when present) of replicated attention parameters
    over the TP group, bucketed; and take the max of the attention-logit telemetry over
    the group, so MuonClip scales the replicated ``k_proj`` identically on every rank."""

    def __init__(self, params: list[Tensor], group: dist.ProcessGroup | None, bucket_bytes: int = 64 << 20,
                 attn_modules: list[nn.Module] | None = None) -> None:
        self.params, self.group, self.bucket_bytes = params, group, bucket_bytes
        self.attn_modules = attn_modules or []

    @torch.no_grad()
    def __call__(self) -> None:
        logits = [m.max_attn_logit for m in self.attn_modules if hasattr(m, "max_attn_logit")]
        if logits:
            flat = torch.stack([x.float() for x in logits])
            dist.all_reduce(flat, op=dist.ReduceOp.MAX, group=self.group)
            for x, v in zip(logits, flat, strict=True):
                x.copy_(v)
        grads = [g for p in self.params if (g := getattr(p, "main_grad", None) if hasattr(p, "main_grad")
                                             else p.grad) is not None]
        i = 0
        while i < len(grads):
            bucket, size = [], 0
            while i < len(grads) and (not bucket or size < self.bucket_bytes):
                bucket.append(grads[i])
                size += grads[i].numel() * grads[i].element_size()
                i += 1
            flat = torch.cat([x.reshape(-1).float() for x in bucket])
            dist.all_reduce(flat, group=self.group)
            off = 0
            for x in bucket:
                x.copy_(flat[off:off + x.numel()].view_as(x))
                off += x.numel()


def apply_tensor_parallel(model: nn.Module, group: dist.ProcessGroup | None = None, *,
                          transport: str = "nccl", max_tokens: int | None = None,
                          timeout_s: float = 30.0) -> TPGradSync:
    """Shard the heads of every block's attention over ``group``; returns the gradient sync
    of the replicated attention parameters (call it after backward, before the optimizer).

    ``transport``: "nccl" (autograd all-reduces through ``torch.distributed``) or "p2p" (the
    NVLink peer-memory kernels of ``parallel.tp_p2p``; CUDA, bf16 activations, one node;
    ``max_tokens`` sizes the receive buffer: tokens per rank per call)."""
    comm = None
    if transport == "p2p":
        from saint_llm_b200.parallel.tp_p2p import PeerTPComm

        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise ValueError("the p2p TP transport needs CUDA parameters")
        if max_tokens is None:
            raise ValueError("the p2p TP transport needs max_tokens (tokens per rank per call)")
        hidden = model.cfg.hidden_dim  # type: ignore[attr-defined]
        comm = PeerTPComm.create(group, dev, max_tokens * hidden, timeout_s=timeout_s)
    elif transport != "nccl":
        raise ValueError(f"unknown TP transport {transport!r}")
    replicated: list[Tensor] = []
    mods = []
    for block in model.blocks:  # type: ignore[attr-defined]
        replicated += shard_attention_heads(block.attention, group, comm)
        mods.append(block.attention)
    sync = TPGradSync(replicated, group, attn_modules=mods)
    sync.comm = comm  # type: ignore[attr-defined]
    return sync


__all__ = ["ColumnParallelLinear", "RowParallelLinear", "TPGradSync", "all_gather_seq", "apply_tensor_parallel",
           "copy_to_tp", "gather_batch_tp", "reduce_from_tp", "reduce_scatter_seq", "shard_attention_heads",
           "split_batch_tp", "split_moe_batches"]

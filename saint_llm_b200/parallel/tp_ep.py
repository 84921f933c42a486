"""Tensor parallelism on attention composed with expert parallelism and (hybrid ZeRO) data
parallelism: the layout of the config-3 brief ("EP=8 + hybrid ZeRO + TP=2 on attention").
The reference has neither TP nor this composition (its multi-GPU path is FSDP2,
``distributed/src/saint_llm_distributed/__init__.py:9-13``).

Layout over a group of W ranks with TP size t: rank ``r`` is TP rank ``r % t`` of replica
``r // t``.  The t ranks of a replica hold the same sequences.

* attention: heads sharded over the replica's TP group (``parallel.tp``);
* MoE layers: each TP rank routes its 1/t of the replica's sequences, and the layer's output
  is gathered over the TP group, so every token reaches the experts once;
* routed experts: sharded over all W ranks (EP = W), token exchange as in ``parallel.ep``;
* everything else: replicated on all W ranks.

Gradients (the loss of a step is the mean over the W / t replicas):

* replicated parameters computed identically by a replica's TP ranks (embedding, mHC, final
  norm, ...): mean over W, as in plain data parallelism;
* partial sums over the TP ranks (replicated attention parameters see only the local heads;
  MoE router / norm / shared experts see only the local sequences): mean over W times t;
* head-sharded attention weights: mean over the replicas holding the same slice, updated on
  every rank (outside ZeRO); Muon orthogonalises the whole matrix (``optim.muon``);
* expert weights: the sum over every rank's tokens divided by W / t.

Data: ``TPEPLayout.replica`` / ``replicas`` name the shard of the global batch a rank reads
(TP ranks of one replica read the same one).

Decoding uses the same layout without gradient state (``shard_for_inference`` +
``parallel_decode``): config 5's TP x EP serving layout.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor, nn

from saint_llm_b200.infer.sampling import SamplingParams
from saint_llm_b200.parallel.ep import ParallelSync, setup_expert_parallel
from saint_llm_b200.parallel.tp import shard_attention_heads, split_moe_batches


@dataclass
class TPEPLayout:
    tp: int
    replicas: int
    replica: int
    tp_rank: int
    tp_group: dist.ProcessGroup | None
    dp_group: dist.ProcessGroup | None


def tp_dp_groups(tp: int, group: dist.ProcessGroup | None = None) -> TPEPLayout:
    """Create the TP groups (consecutive ranks) and the slice groups (ranks with the same TP
    index) of ``group``; every rank of ``group`` must call this, in the same order."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if tp < 1 or world % tp:
        raise ValueError(f"TP size {tp} must divide the group size {world}")
    glob = [dist.get_global_rank(group, r) if group is not None else r for r in range(world)]
    tp_group = dp_group = None
    for rep in range(world // tp):
        g = dist.new_group([glob[rep * tp + i] for i in range(tp)])
        if rank // tp == rep:
            tp_group = g
    for i in range(tp):
        g = dist.new_group([glob[rep * tp + i] for rep in range(world // tp)])
        if rank % tp == i:
            dp_group = g
    return TPEPLayout(tp, world // tp, rank // tp, rank % tp, tp_group, dp_group)


def setup_tp_ep(model: nn.Module, tp: int, group: dist.ProcessGroup | None = None, *, transport: str = "auto",
                zero: bool = False, overlap_reduce: bool = False, zero_transport: str = "nccl",
                timeout_s: float = 30.0, tp_transport: str = "nccl", max_tokens: int | None = None,
                capacity_factor: float | None = None) -> tuple[ParallelSync, TPEPLayout]:
    """Shard ``model`` as described in the module docstring; returns the gradient
    synchroniser (use it like ``setup_expert_parallel``'s: ``sync(params)`` after the
    backward, ``configure_optimizer`` once, ``post_step`` after the optimizer) and the layout.

    ``tp_transport``: "nccl" (autograd all-reduces) or "p2p" (the NVLink peer-memory kernels
    of ``parallel.tp_p2p``; ``max_tokens`` = tokens per rank per call)."""
    lay = tp_dp_groups(tp, group)
    comm = None
    if tp_transport == "p2p":
        from saint_llm_b200.parallel.tp_p2p import PeerTPComm

        dev = next(model.parameters()).device
        if dev.type != "cuda" or max_tokens is None:
            raise ValueError("the p2p TP transport needs CUDA parameters and max_tokens")
        comm = PeerTPComm.create(lay.tp_group, dev, max_tokens * model.cfg.hidden_dim,  # type: ignore[attr-defined]
                                 timeout_s=timeout_s)
    elif tp_transport != "nccl":
        raise ValueError(f"unknown TP transport {tp_transport!r}")
    partial: list = []
    sharded: list = []
    shards: dict[int, tuple[object, int]] = {}
    for block in model.blocks:  # type: ignore[attr-defined]
        attn = block.attention
        rep = shard_attention_heads(attn, lay.tp_group, comm)
        ids = {id(p) for p in rep}
        partial += rep
        sharded += [p for p in attn.parameters() if id(p) not in ids and p.requires_grad]
        shards[id(attn.q_up.weight)] = (lay.tp_group, 0)             # rows: local heads
        shards[id(attn.output.final_proj.weight)] = (lay.tp_group, 1)  # columns: local groups
    for moe in split_moe_batches(model, lay.tp_group):
        partial += [p for n, p in moe.named_parameters() if not n.startswith("grouped_experts.") and p.requires_grad]
    sync = setup_expert_parallel(model, group, transport=transport, capacity_factor=capacity_factor, zero=zero,
                                 timeout_s=timeout_s, overlap_reduce=overlap_reduce, zero_transport=zero_transport,
                                 dp_params=sharded, dp_group=lay.dp_group, partial_params=partial,
                                 partial_scale=float(tp), expert_div=lay.replicas)
    sync.tp_shards = shards
    sync.tp_comm = comm  # type: ignore[attr-defined]
    return sync, lay


def shard_for_inference(model: nn.Module, tp: int, group: dist.ProcessGroup | None = None) -> TPEPLayout:
    """The same layout for decoding (config 5's TP x EP): heads over each TP group, the routed
    experts over all ranks, each TP rank routing its share of the batch (the decode batch of a
    replica must divide by ``tp``).  Every rank of ``group`` calls this; no gradient state."""
    from saint_llm_b200.parallel.ep import shard_grouped_experts

    lay = tp_dp_groups(tp, group)
    for block in model.blocks:  # type: ignore[attr-defined]
        shard_attention_heads(block.attention, lay.tp_group)
    split_moe_batches(model, lay.tp_group)
    shard_grouped_experts(model, dist.get_rank(group), dist.get_world_size(group), group)
    return lay


def parallel_decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int,
                    params: SamplingParams | None = None, eos_token: int | None = None,
                    generator: torch.Generator | None = None, use_cache: bool = True) -> Tensor:
    """``infer.generate.decode`` for a model sharded by ``shard_for_inference``: this rank's
    replica decodes ``prompt_ids`` (the TP ranks of a replica pass the same prompts and, for
    sampling, identically seeded generators).  The expert exchange is a collective over all
    ranks, so every rank runs all ``max_new_tokens`` steps: rows that produced ``eos_token``
    are filled with it afterwards instead of ending the loop early (the output is the same)."""
    from saint_llm_b200.infer.generate import decode

    out = decode(model, prompt_ids, max_new_tokens=max_new_tokens, params=params or SamplingParams(),
                 generator=generator, use_cache=use_cache)
    if eos_token is not None:
        gen = out[:, prompt_ids.shape[1]:]
        hit = (gen == eos_token).long().cumsum(1) > 0
        gen.masked_fill_(hit, eos_token)
    return out


__all__ = ["TPEPLayout", "parallel_decode", "setup_tp_ep", "shard_for_inference", "tp_dp_groups"]

"""DeepSeekMoE: shared experts + hash/learned-routed experts with SwiGLU.

Semantics (reference ``core/moe.py:31-242``):

* ``SwiGLU``: ``down(silu(min(gate(x), g_max)) * clamp(up(x), lo, hi))``.
* ``HashRouter``: ``h <- (h * 2654435769 + j * 0x9E3779B9) mod 2^31`` per slot j,
  expert ``h mod E``; a slot colliding with an earlier slot moves to ``(e+1) mod E``;
  weights 1/k.
* ``LearnedRouter``: affinity ``sqrt(softplus(W x) + 1e-12)`` (or sigmoid); top-k on
  ``affinity + aux_free_bias (+ modality_bias[is_visual])``; gates renormalised from
  the *unbiased* affinity.
* Sequence balance loss ``E * sum_e freq_e * mean_aff_e`` (mean over batch).
* Output = sum of shared experts + gate-weighted routed experts.

The reference never updates ``aux_free_bias``; ``LearnedRouter.update_bias`` adds
the DeepSeek-V3 aux-loss-free rule (``b += speed * sign(mean_load - load)``) behind
the ``update_aux_free_bias`` flag, default off (reference behaviour).

On CUDA the layer runs ``ops.moe.moe_forward`` (fused router + top-k, expert-sorted
permutation, grouped tensor-core GEMMs with the SwiGLU/clamp epilogue, gate-weighted
combine); the shared experts ride in the same grouped GEMM as always-selected
experts.  With expert parallelism the dispatch/combine go over NVLink inside the
same path (``parallel.ep``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.config import MoEConfig
from saint_llm_b200.models.attention.common import RMSNorm
from saint_llm_b200.models.linear import LinearFactory, default_linear
from saint_llm_b200.ops import backend

_HASH_MULT = 2654435769
_HASH_STEP = 0x9E3779B9
_HASH_MOD = 2**31


class SwiGLU(nn.Module):
    def __init__(self, hidden_dim: int, intermediate_dim: int, clamp_linear: tuple[float, float],
                 clamp_gate_max: float, *, linear_factory: LinearFactory = default_linear) -> None:
        super().__init__()
        self.gate_proj = linear_factory(hidden_dim, intermediate_dim, bias=False)
        self.up_proj = linear_factory(hidden_dim, intermediate_dim, bias=False)
        self.down_proj = linear_factory(intermediate_dim, hidden_dim, bias=False)
        self.clamp_linear = clamp_linear
        self.clamp_gate_max = clamp_gate_max

    def forward(self, x: Tensor) -> Tensor:
        g = self.gate_proj(x).clamp(max=self.clamp_gate_max)
        u = self.up_proj(x).clamp(min=self.clamp_linear[0], max=self.clamp_linear[1])
        return self.down_proj(F.silu(g) * u)


class HashRouter:
    @staticmethod
    def route(token_ids: Tensor, n_experts: int, k: int) -> tuple[Tensor, Tensor]:
        h = token_ids.long()
        cols = []
        for j in range(k):
            h = (h * _HASH_MULT + j * _HASH_STEP) % _HASH_MOD
            cols.append(h % n_experts)
        idx = torch.stack(cols, dim=-1)
        for j in range(1, k):
            clash = (idx[..., j : j + 1] == idx[..., :j]).any(-1)
            idx[..., j] = torch.where(clash, (idx[..., j] + 1) % n_experts, idx[..., j])
        return idx, torch.full(idx.shape, 1.0 / k, dtype=torch.float32, device=idx.device)


class LearnedRouter(nn.Module):
    def __init__(self, hidden_dim: int, n_routed: int, top_k: int, cfg: MoEConfig,
                 enable_modality_bias: bool) -> None:
        super().__init__()
        self.n_routed = n_routed
        self.top_k = top_k
        self.cfg = cfg
        self.score_proj = nn.Linear(hidden_dim, n_routed, bias=False)
        self.register_buffer("aux_free_bias", torch.zeros(n_routed))
        self.modality_bias: nn.Parameter | None = (
            nn.Parameter(torch.zeros(2, n_routed)) if enable_modality_bias else None
        )
        self.update_aux_free_bias = False

    def affinity(self, x: Tensor) -> Tensor:
        if backend.native_for(x):
            from saint_llm_b200.ops.linear import linear

            logits = linear(x, self.score_proj.weight).float()
        else:
            logits = self.score_proj(x)
        if self.cfg.affinity_fn == "sqrt_softplus":
            return torch.sqrt(F.softplus(logits) + 1.0e-12)
        return torch.sigmoid(logits)

    def forward(self, x: Tensor, is_visual: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
        if backend.native_for(x) and self.n_routed <= 256 and self.top_k <= 16:
            from saint_llm_b200.ops.linear import linear
            from saint_llm_b200.ops.router import fused_route

            logits = linear(x, self.score_proj.weight).float()
            return fused_route(logits, self.top_k, self.cfg.affinity_fn, self.aux_free_bias,
                               self.modality_bias, is_visual)
        aff = self.affinity(x)
        biased = aff + self.aux_free_bias
        if self.modality_bias is not None and is_visual is not None:
            biased = biased + self.modality_bias[is_visual.long()]
        _, idx = biased.topk(self.top_k, dim=-1)
        g = aff.gather(-1, idx)
        return idx, g / (g.sum(-1, keepdim=True) + 1.0e-12), aff

    @torch.no_grad()
    def update_bias(self, expert_counts: Tensor) -> None:
        """Aux-loss-free balancing step from per-expert token counts of the last batch."""
        load = expert_counts.float()
        self.aux_free_bias.add_(self.cfg.aux_loss_free_bias_speed * torch.sign(load.mean() - load))


def sequence_balance_loss(affinity: Tensor, expert_idx: Tensor) -> Tensor:
    n = affinity.shape[-1]
    b, t, k = expert_idx.shape
    counts = torch.zeros(b, n, device=affinity.device, dtype=torch.float32)
    counts.scatter_add_(1, expert_idx.reshape(b, t * k), torch.ones(b, t * k, device=affinity.device))
    freq = counts / (t * k)
    return (freq * affinity.mean(dim=1)).sum(-1).mean() * n


def sharded_balance_loss(affinity: Tensor, expert_idx: Tensor, group: object) -> Tensor:
    """``sequence_balance_loss`` of sequences whose tokens are split over ``group`` (context
    parallelism): the per-sequence expert counts and affinity sums are summed over the group
    (the affinity sum through a differentiable all-reduce), and this rank returns its 1/ws
    share, so the shares add up to the loss of the whole sequences and so do the gradients."""
    import torch.distributed as dist
    from torch.distributed.nn.functional import all_reduce

    n = affinity.shape[-1]
    b, t, k = expert_idx.shape
    ws = dist.get_world_size(group)
    counts = torch.zeros(b, n, device=affinity.device, dtype=torch.float32)
    counts.scatter_add_(1, expert_idx.reshape(b, t * k), torch.ones(b, t * k, device=affinity.device))
    dist.all_reduce(counts, group=group)
    total = t * ws
    aff_sum = all_reduce(affinity.float().sum(dim=1), group=group)
    return ((counts / (total * k)) * (aff_sum / total)).sum(-1).mean() * n / ws


class DeepSeekMoE(nn.Module):
    def __init__(self, hidden_dim: int, cfg: MoEConfig, layer_idx: int,
                 enable_modality_router_bias: bool = True, *,
                 linear_factory: LinearFactory = default_linear, use_grouped_gemm: bool = False,
                 grouped_quant: str = "bf16", fp4_block_size: int = 32) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.use_grouped_gemm = use_grouped_gemm
        self.use_hash_routing = layer_idx < cfg.hash_routed_layers
        self.norm = RMSNorm(hidden_dim)
        mk = lambda: SwiGLU(hidden_dim, cfg.expert_intermediate_dim, cfg.swiglu_clamp_linear,  # noqa: E731
                            cfg.swiglu_clamp_gate_max, linear_factory=linear_factory)
        self.shared_experts = nn.ModuleList(mk() for _ in range(cfg.shared_experts))
        self.grouped_experts: nn.Module | None
        if use_grouped_gemm:
            from saint_llm_b200.ops.moe import GroupedSwiGLUExperts

            self.grouped_experts = GroupedSwiGLUExperts(
                hidden_dim, cfg.expert_intermediate_dim, cfg.routed_experts,
                clamp_linear=cfg.swiglu_clamp_linear, clamp_gate_max=cfg.swiglu_clamp_gate_max,
                linear_quant=grouped_quant, fp4_block_size=fp4_block_size,
            )
            self.routed_experts = nn.ModuleList()
        else:
            self.grouped_experts = None
            self.routed_experts = nn.ModuleList(mk() for _ in range(cfg.routed_experts))
        self.router: LearnedRouter | None = (
            None if self.use_hash_routing else LearnedRouter(
                hidden_dim, cfg.routed_experts, cfg.experts_per_token, cfg,
                enable_modality_bias=enable_modality_router_bias)
        )
        self._last_aux_loss: Tensor | None = None
        self.register_buffer("last_expert_counts", torch.zeros(cfg.routed_experts), persistent=False)
        # expert parallelism (set by parallel.ep.shard_grouped_experts); None = all experts local
        self.ep_group = None
        self.ep_size = 1
        self.ep_rank = 0
        # tensor parallelism (set by parallel.tp.split_moe_batches): the TP ranks hold the same
        # sequences; each routes its own 1/tp of them and the outputs are gathered
        self.tp_group = None
        self.tp_size = 1
        self.tp_rank = 0
        # context parallelism (set for the duration of a CP forward by parallel.cp.balance_over):
        # the sequences are sharded over this group, so the balance loss pools its statistics
        self.balance_group = None

    def route(self, h: Tensor, token_ids: Tensor | None, is_visual: Tensor | None
              ) -> tuple[Tensor, Tensor, Tensor]:
        """(expert_idx (B,T,k), gates (B,T,k) fp32, aux loss scalar)."""
        if self.use_hash_routing:
            if token_ids is None:
                raise ValueError("hash-routed MoE layers need token_ids")
            idx, gate = HashRouter.route(token_ids, self.cfg.routed_experts, self.cfg.experts_per_token)
            return idx, gate, h.new_zeros(())
        assert self.router is not None
        idx, gate, aff = self.router(h, is_visual=is_visual)
        if self.balance_group is not None:
            return idx, gate, sharded_balance_loss(aff, idx, self.balance_group)
        return idx, gate, sequence_balance_loss(aff, idx)

    def forward(self, x: Tensor, token_ids: Tensor | None = None,
                is_visual: Tensor | None = None) -> Tensor:
        if self.tp_size > 1:
            return self._forward_tp_split(x, token_ids, is_visual)
        return self._forward_local(x, token_ids, is_visual)

    def _forward_tp_split(self, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
        """This TP rank's share of the batch through the layer, then the shares gathered.  The
        balance loss of a share is scaled by 1/tp: summed over the TP group (as its router
        gradients are) it is the batch mean of the unsplit layer."""
        from saint_llm_b200.parallel.tp import gather_batch_tp, split_batch_tp

        b = x.shape[0]
        if b % self.tp_size:
            raise ValueError(f"batch {b} not divisible by the TP size {self.tp_size}")
        n = b // self.tp_size
        rows = slice(self.tp_rank * n, (self.tp_rank + 1) * n)
        y = self._forward_local(split_batch_tp(x, self.tp_group), None if token_ids is None else token_ids[rows],
                                None if is_visual is None else is_visual[rows])
        if self._last_aux_loss is not None:
            self._last_aux_loss = self._last_aux_loss / self.tp_size
        return gather_batch_tp(y, self.tp_group)

    def _forward_local(self, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
        if self.ep_size > 1:
            from saint_llm_b200.parallel import ep

            return ep.moe_forward_ep(self, x, token_ids, is_visual)
        if backend.native_for(x):
            from saint_llm_b200.ops import moe as moe_ops

            return moe_ops.moe_forward(self, x, token_ids, is_visual)
        h = self.norm(x)
        b, t, d = h.shape
        idx, gate, aux = self.route(h, token_ids, is_visual)
        self._last_aux_loss = aux
        k = self.cfg.experts_per_token
        fh, fi, fg = h.reshape(b * t, d), idx.reshape(b * t, k), gate.reshape(b * t, k)
        with torch.no_grad():
            self.last_expert_counts.copy_(torch.bincount(fi.reshape(-1), minlength=self.cfg.routed_experts))
        if self.grouped_experts is not None:
            routed = self.grouped_experts(fh, fi, fg).reshape(b, t, d)
        else:
            routed = torch.zeros_like(h)
            flat_routed = routed.view(b * t, d)
            for e, expert in enumerate(self.routed_experts):
                tok, slot = (fi == e).nonzero(as_tuple=True)
                if tok.numel() == 0:
                    continue
                flat_routed.index_add_(0, tok, expert(fh[tok]) * fg[tok, slot].unsqueeze(-1).to(fh.dtype))
        shared = torch.zeros_like(h)
        for expert in self.shared_experts:
            shared = shared + expert(h)
        return shared + routed

    @staticmethod
    def _sequence_balance_loss(affinity: Tensor, expert_idx: Tensor) -> Tensor:
        return sequence_balance_loss(affinity, expert_idx)


__all__ = ["DeepSeekMoE", "HashRouter", "LearnedRouter", "SwiGLU", "sequence_balance_loss", "sharded_balance_loss"]

"""``SaintLLM``: the V4-style model (reference ``core/model.py:71-352``).

embed -> modality splice -> (sinks at prefill) -> mHC expand -> blocks -> mHC collapse
-> drop sinks -> final RMSNorm -> tied LM head (-> softcap) ; MTP hidden states ->
tied head ; generation head ; summed MoE aux loss.

Each block: attention (SWA for ``idx < first_dense_swa_layers``, else CSA/HCA
alternating) and MoE, each wrapped in its own mHC.  Parameter names and shapes are
those of the reference, so checkpoints load in both directions.

Differences that do not change results:
* telemetry (max attention logit, expert counts) stays on the device -- the
  reference syncs the host in every attention layer and every block;
* on CUDA the sub-layers dispatch to the fused sm_100a kernels;
* ``forward(..., return_hidden_only=True)`` skips the vocabulary projection so the
  fused LM-head cross-entropy (``ops.ce``) can consume the hidden states directly.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from saint_llm_b200.config import ModelConfig
from saint_llm_b200.models.attention import CSA, HCA, NSAttention, RMSNorm, SWAttention
from saint_llm_b200.models.init import normal_init, umup_init
from saint_llm_b200.models.linear import LinearFactory, make_linear_factory
from saint_llm_b200.models.mhc import MHC
from saint_llm_b200.models.moe import DeepSeekMoE
from saint_llm_b200.models.mtp import MTPStack
from saint_llm_b200.models.multimodal import GenerationHeadHook, ModalityProjector, ResidualSideChannel
from saint_llm_b200.ops import backend


def _apply_linear(mod: nn.Linear, x: Tensor) -> Tensor:
    from saint_llm_b200.ops import backend

    if backend.native_for(x):
        from saint_llm_b200.ops.linear import linear

        return linear(x, mod.weight, mod.bias)
    return mod(x)


class TransformerBlock(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_idx: int, *, linear_factory: LinearFactory) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        kind = cfg.layer_kind(layer_idx)
        self.attention: nn.Module
        if kind == "swa":
            self.attention = SWAttention(cfg.hidden_dim, cfg.attention, linear_factory=linear_factory)
        elif kind == "csa":
            self.attention = CSA(cfg.hidden_dim, cfg.attention, cfg.csa, linear_factory=linear_factory)
        elif kind == "nsa":
            self.attention = NSAttention(cfg.hidden_dim, cfg.attention, compression_rate=cfg.nsa.compression_rate,
                                         selection_k=cfg.nsa.selection_k, linear_factory=linear_factory)
        else:
            self.attention = HCA(cfg.hidden_dim, cfg.attention, cfg.hca, linear_factory=linear_factory)
        self.attn_mhc = MHC(cfg.hidden_dim, cfg.mhc, rms_norm_eps=cfg.rms_norm_eps)
        self.moe_mhc = MHC(cfg.hidden_dim, cfg.mhc, rms_norm_eps=cfg.rms_norm_eps)
        self.moe = DeepSeekMoE(
            cfg.hidden_dim, cfg.moe, layer_idx=layer_idx,
            enable_modality_router_bias=cfg.multimodal.enable_modality_router_bias,
            linear_factory=linear_factory, use_grouped_gemm=cfg.moe_use_grouped_gemm,
            grouped_quant=cfg.linear_quant, fp4_block_size=cfg.fp4_block_size,
        )
        self.side_channel = ResidualSideChannel(cfg.hidden_dim, cfg.multimodal.side_channel_alpha_init)

    def forward(self, x: Tensor, token_ids: Tensor, is_visual: Tensor | None, *,
                kv_cache_layer: object | None = None) -> Tensor:
        inner, _, b_l, c_l = self.attn_mhc.split(x)
        if kv_cache_layer is not None:
            a = self.attention(inner, is_visual=is_visual, kv_cache=kv_cache_layer)
        else:
            a = self.attention(inner, is_visual=is_visual)
        x = self.attn_mhc.combine(x, a, b_l, c_l)
        inner, _, b_l, c_l = self.moe_mhc.split(x)
        x = self.moe_mhc.combine(x, self.moe(inner, token_ids=token_ids, is_visual=is_visual), b_l, c_l)
        if self.side_channel.active:
            collapsed = x.mean(-2)
            x = x + ((self.side_channel(collapsed) - collapsed) / x.shape[-2]).unsqueeze(-2)
        return x


class SaintLLM(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_dim)
        mm = cfg.multimodal
        self.vision_proj = ModalityProjector(mm.vision_input_dim, cfg.hidden_dim, enabled=mm.enable_vision_projector)
        self.audio_proj = ModalityProjector(mm.audio_input_dim, cfg.hidden_dim, enabled=mm.enable_audio_projector)
        factory = make_linear_factory(cfg.linear_quant, fp4_block_size=cfg.fp4_block_size,
                                      fp8_use_real_gemm=cfg.fp8_use_real_gemm)
        self.blocks = nn.ModuleList(TransformerBlock(cfg, i, linear_factory=factory) for i in range(cfg.n_layers))
        self.final_norm = RMSNorm(cfg.hidden_dim, eps=cfg.rms_norm_eps)
        self.lm_head = nn.Linear(cfg.hidden_dim, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.embed.weight
        self.mtp = MTPStack(cfg.hidden_dim, cfg.vocab_size, cfg.mtp, rms_norm_eps=cfg.rms_norm_eps)
        self.generation_head = GenerationHeadHook(cfg.hidden_dim, mm.generation_head_vocab,
                                                  enabled=mm.enable_generation_head)
        self.sink_embeddings: nn.Parameter | None = (
            nn.Parameter(torch.randn(cfg.n_sink_tokens, cfg.hidden_dim) / math.sqrt(cfg.hidden_dim))
            if cfg.n_sink_tokens > 0 else None
        )
        self._init_weights()

    def _init_weights(self) -> None:
        if self.cfg.init_scheme == "umup":
            umup_init(self, n_layers=self.cfg.n_layers)
        else:
            normal_init(self, self.cfg.initializer_range)

    # ---- inputs ------------------------------------------------------------------
    def _embed_inputs(self, token_ids: Tensor, vision_features: Tensor | None,
                      audio_features: Tensor | None) -> Tensor:
        if backend.native_for(self.embed.weight):
            from saint_llm_b200.ops.embedding import embedding

            h = embedding(token_ids, self.embed.weight)
        else:
            h = self.embed(token_ids)
        slots, mm = self.cfg.tokenizer_slots, self.cfg.multimodal
        if vision_features is not None and mm.enable_vision_projector:
            mask = token_ids == slots.image_pad
            n = int(mask.sum())
            if n > 0:
                if vision_features.shape[0] != n:
                    raise ValueError(f"vision_features has {vision_features.shape[0]} rows but token "
                                     f"sequence has {n} <|image_pad|> slots — must match")
                h = h.clone()
                h[mask] = self.vision_proj(vision_features).to(h.dtype)
        if audio_features is not None and mm.enable_audio_projector:
            mask = (token_ids >= slots.audio_start) & (token_ids <= slots.audio_end)
            n = int(mask.sum())
            if n > 0:
                if audio_features.shape[0] != n:
                    raise ValueError(f"audio_features has {audio_features.shape[0]} rows but token "
                                     f"sequence has {n} audio slots — must match")
                h = h.clone()
                h[mask] = self.audio_proj(audio_features).to(h.dtype)
        return h

    def backbone(self, token_ids: Tensor, vision_features: Tensor | None = None,
                 audio_features: Tensor | None = None, is_visual: Tensor | None = None, *,
                 kv_cache_bundle: object | None = None) -> tuple[Tensor, Tensor]:
        """Final-normed hidden states (B, T, D) and input embeddings (B, T, D)."""
        h = self._embed_inputs(token_ids, vision_features, audio_features)
        emb = h
        if is_visual is None:
            is_visual = token_ids == self.cfg.tokenizer_slots.image_pad
        n_sink = self.cfg.n_sink_tokens
        warm = kv_cache_bundle is not None and getattr(kv_cache_bundle, "length", 0) > 0
        sinks = self.sink_embeddings is not None and n_sink > 0 and not warm
        ids, vis = token_ids, is_visual
        if sinks:
            b = h.shape[0]
            assert self.sink_embeddings is not None
            h = torch.cat([self.sink_embeddings.to(h.dtype).unsqueeze(0).expand(b, n_sink, -1), h], dim=1)
            ids = torch.cat([token_ids.new_zeros(b, n_sink), token_ids], dim=1)
            vis = torch.cat([is_visual.new_zeros(b, n_sink), is_visual], dim=1)
        x = MHC.expand(h, self.cfg.mhc.expansion_factor)
        ckpt = self.cfg.activation_checkpointing and self.training and torch.is_grad_enabled()
        for i, block in enumerate(self.blocks):
            if ckpt and kv_cache_bundle is None:
                x = checkpoint(lambda t, blk=block: blk(t, token_ids=ids, is_visual=vis), x,
                               use_reentrant=False)
            else:
                layer_cache = kv_cache_bundle.for_layer(i) if kv_cache_bundle is not None else None  # type: ignore[attr-defined]
                x = block(x, token_ids=ids, is_visual=vis, kv_cache_layer=layer_cache)
        h = MHC.collapse(x)
        if sinks:
            h = h[:, n_sink:]
        return self.final_norm(h), emb

    def logits(self, h: Tensor) -> Tensor:
        out = _apply_linear(self.lm_head, h)
        c = self.cfg.final_logit_softcap
        return c * torch.tanh(out / c) if c is not None else out

    def aux_loss(self) -> Tensor | None:
        total: Tensor | None = None
        for block in self.blocks:
            a = getattr(block.moe, "_last_aux_loss", None)
            if isinstance(a, Tensor):
                total = a if total is None else total + a
        return total

    def forward(self, token_ids: Tensor, vision_features: Tensor | None = None,
                audio_features: Tensor | None = None, is_visual: Tensor | None = None, *,
                kv_cache_bundle: object | None = None,
                return_hidden_only: bool = False) -> dict[str, Tensor | list[Tensor] | None]:
        h, emb = self.backbone(token_ids, vision_features, audio_features, is_visual,
                               kv_cache_bundle=kv_cache_bundle)
        mtp_hidden = self.mtp(h, emb)
        if return_hidden_only:
            return {"hidden": h, "mtp_hidden": mtp_hidden, "aux_loss": self.aux_loss(),
                    "logits": None, "mtp_logits": None, "generation_logits": None}
        return {
            "logits": self.logits(h),
            "mtp_logits": [self.logits(mh) for mh in mtp_hidden],
            "generation_logits": _apply_linear(self.generation_head.proj, h),
            "hidden": h,
            "aux_loss": self.aux_loss(),
        }

    # ---- utilities ---------------------------------------------------------------
    def attention_layers(self) -> list[nn.Module]:
        return [b.attention for b in self.blocks]

    def num_parameters(self, *, active_only: bool = False) -> int:
        seen: set[int] = set()
        total = 0
        for name, p in self.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            n = p.numel()
            if active_only and (".routed_experts." in name or ".grouped_experts." in name):
                moe = self.cfg.moe
                n = n * moe.experts_per_token // moe.routed_experts
            total += n
        return total


__all__ = ["SaintLLM", "TransformerBlock"]

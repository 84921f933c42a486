"""Model and run configuration.

``ModelConfig`` and its sub-configs keep the reference's field names, defaults and
presets so a reference config (and checkpoint) maps 1:1 onto this framework
(reference: ``core/config.py:14-284``).  Everything that is about *how* the model
runs on B200s -- parallel layout, precision recipe, kernel toggles, timeouts -- lives
in the separate :class:`RunConfig`, never in ``ModelConfig``.

The five benchmark configurations of the project brief are exposed as
``ModelConfig.bench_tiny()`` ... ``ModelConfig.bench_decode()`` with every field the
brief leaves open pinned explicitly (documented on each preset).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Literal

from pydantic import BaseModel, ConfigDict, Field


class _Frozen(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")


class CSAConfig(_Frozen):
    """Compressed sparse attention: compression rate m, lightning-indexer shape, top-k."""

    compression_rate: int = 4
    indexer_query_heads: int = 64
    indexer_head_dim: int = 128
    attention_top_k: int = 512


class NSAConfig(_Frozen):
    compression_rate: int = 32
    selection_k: int = 16


class HCAConfig(_Frozen):
    """Heavily compressed attention: compression rate m'."""

    compression_rate: int = 128


class AttentionConfig(_Frozen):
    query_heads: int = 64
    head_dim: int = 512
    query_compression_dim: int = 1024
    output_proj_groups: int = 8
    attention_intermediate_dim: int = 1024
    sliding_window_size: int = 128
    rope_dim: int = 64
    rope_theta: float = 10000.0
    use_attention_sink: bool = True
    logit_softcap: float | None = None


class MoEConfig(_Frozen):
    hash_routed_layers: int = 3
    shared_experts: int = 1
    routed_experts: int = 256
    experts_per_token: int = 6
    expert_intermediate_dim: int = 2048
    affinity_fn: Literal["sqrt_softplus", "sigmoid"] = "sqrt_softplus"
    aux_loss_free_bias_speed: float = 0.001
    sequence_balance_weight: float = 0.0001
    swiglu_clamp_linear: tuple[float, float] = (-10.0, 10.0)
    swiglu_clamp_gate_max: float = 10.0


class MHCConfig(_Frozen):
    expansion_factor: int = 4
    sinkhorn_iters: int = 20
    init_alpha: float = 0.02
    init_static_bias: float = 0.0


class MTPConfig(_Frozen):
    depth: int = 1
    loss_weight_main: float = 0.3
    loss_weight_decay: float = 0.1


class MultimodalConfig(_Frozen):
    enable_vision_projector: bool = False
    vision_input_dim: int = 1152
    enable_audio_projector: bool = False
    audio_input_dim: int = 1280
    enable_mrope: bool = False
    enable_residual_side_channel: bool = True
    side_channel_alpha_init: float = 0.0
    enable_generation_head: bool = False
    generation_head_vocab: int = 2368
    enable_modality_router_bias: bool = True


class TokenizerSlots(_Frozen):
    image_pad: int = 128514
    audio_start: int = 128518
    audio_end: int = 128519
    video_start: int = 128515
    video_end: int = 128516
    think_start: int = 128648
    think_end: int = 128649
    memory_block_base: int = 128710


def _small_slots(base: int) -> TokenizerSlots:
    """Control-token ids packed right below ``base`` (for small vocabularies)."""
    return TokenizerSlots(
        image_pad=base, audio_start=base + 1, audio_end=base + 5, video_start=base + 6,
        video_end=base + 7, think_start=base + 8, think_end=base + 9, memory_block_base=base + 10,
    )


class ModelConfig(_Frozen):
    variant: Literal["flash", "pro"] = "flash"
    n_layers: int = 43
    hidden_dim: int = 4096
    vocab_size: int = 131072

    first_dense_swa_layers: int = 2
    # "nsa" (an extension): every layer after the dense SWA layers is NSA
    attention_pattern: Literal["csa_hca_interleaved", "nsa"] = "csa_hca_interleaved"

    csa: CSAConfig = Field(default_factory=CSAConfig)
    hca: HCAConfig = Field(default_factory=HCAConfig)
    nsa: NSAConfig = Field(default_factory=NSAConfig)
    attention: AttentionConfig = Field(default_factory=AttentionConfig)
    moe: MoEConfig = Field(default_factory=MoEConfig)
    mhc: MHCConfig = Field(default_factory=MHCConfig)
    mtp: MTPConfig = Field(default_factory=MTPConfig)
    multimodal: MultimodalConfig = Field(default_factory=MultimodalConfig)
    tokenizer_slots: TokenizerSlots = Field(default_factory=TokenizerSlots)

    rms_norm_eps: float = 1.0e-6
    initializer_range: float = 0.02
    tie_word_embeddings: bool = True
    init_scheme: Literal["normal", "umup"] = "normal"
    final_logit_softcap: float | None = None
    n_sink_tokens: int = 0

    linear_quant: Literal["bf16", "fp8", "fp4"] = "bf16"
    fp4_block_size: int = 32
    fp8_use_real_gemm: bool = False
    moe_use_grouped_gemm: bool = False
    activation_checkpointing: bool = False

    # ---- helpers -------------------------------------------------------------------
    def layer_kind(self, layer_idx: int) -> Literal["swa", "csa", "hca", "nsa"]:
        """Attention type of block ``layer_idx`` (SWA first, then CSA/HCA alternating)."""
        if layer_idx < self.first_dense_swa_layers:
            return "swa"
        if self.attention_pattern == "nsa":
            return "nsa"
        return "csa" if (layer_idx - self.first_dense_swa_layers) % 2 == 0 else "hca"

    def to_json(self) -> str:
        return self.model_dump_json()

    @classmethod
    def from_json(cls, text: str) -> ModelConfig:
        return cls.model_validate_json(text)

    # ---- reference presets (core/config.py:161-284) --------------------------------
    @classmethod
    def v4_flash(cls) -> ModelConfig:
        return cls()

    @classmethod
    def v4_pro(cls) -> ModelConfig:
        return cls(
            variant="pro", n_layers=61, hidden_dim=7168,
            csa=CSAConfig(attention_top_k=1024),
            attention=AttentionConfig(query_heads=128, head_dim=512, query_compression_dim=1536,
                                      output_proj_groups=16),
            moe=MoEConfig(routed_experts=384, expert_intermediate_dim=3072),
        )

    @classmethod
    def small_flash(cls, *, vocab_size: int = 32_768) -> ModelConfig:
        return cls(
            variant="flash", n_layers=8, hidden_dim=768, vocab_size=vocab_size,
            first_dense_swa_layers=1,
            csa=CSAConfig(compression_rate=4, indexer_query_heads=4, indexer_head_dim=64,
                          attention_top_k=64),
            hca=HCAConfig(compression_rate=64),
            attention=AttentionConfig(query_heads=12, head_dim=64, query_compression_dim=512,
                                      output_proj_groups=4, attention_intermediate_dim=192,
                                      sliding_window_size=128, rope_dim=32),
            moe=MoEConfig(hash_routed_layers=2, shared_experts=1, routed_experts=4,
                          experts_per_token=2, expert_intermediate_dim=1536),
            mhc=MHCConfig(expansion_factor=2, sinkhorn_iters=8),
            tokenizer_slots=_small_slots(32500),
        )

    @classmethod
    def tiny(cls) -> ModelConfig:
        return cls(
            variant="flash", n_layers=4, hidden_dim=128, vocab_size=512,
            first_dense_swa_layers=1,
            csa=CSAConfig(compression_rate=2, indexer_query_heads=2, indexer_head_dim=16,
                          attention_top_k=8),
            hca=HCAConfig(compression_rate=8),
            attention=AttentionConfig(query_heads=4, head_dim=32, query_compression_dim=32,
                                      output_proj_groups=2, attention_intermediate_dim=32,
                                      sliding_window_size=8, rope_dim=8),
            moe=MoEConfig(hash_routed_layers=1, shared_experts=1, routed_experts=8,
                          experts_per_token=2, expert_intermediate_dim=64),
            mhc=MHCConfig(expansion_factor=2, sinkhorn_iters=5),
            tokenizer_slots=_small_slots(500),
        )

    # ---- benchmark presets (the five configurations of the project brief) ---------
    # Fields the brief leaves open are pinned here and used identically by the
    # reference arm of bench.py: first_dense_swa_layers=0 and hash_routed_layers=0
    # ("CSA alternating HCA", every MoE layer learned-routed); other open fields keep
    # the reference defaults unless noted.
    @classmethod
    def bench_tiny(cls) -> ModelConfig:
        """Config 1: tiny V4 on CPU (vocab 8192, d 256, 4 layers, 8x32 heads)."""
        return cls(
            n_layers=4, hidden_dim=256, vocab_size=8192, first_dense_swa_layers=0,
            csa=CSAConfig(compression_rate=64, indexer_query_heads=4, indexer_head_dim=32,
                          attention_top_k=4),
            hca=HCAConfig(compression_rate=8),
            attention=AttentionConfig(query_heads=8, head_dim=32, query_compression_dim=128,
                                      output_proj_groups=2, attention_intermediate_dim=128,
                                      sliding_window_size=64, rope_dim=16),
            moe=MoEConfig(hash_routed_layers=0, shared_experts=1, routed_experts=8,
                          experts_per_token=2, expert_intermediate_dim=512),
            mhc=MHCConfig(expansion_factor=2),
            mtp=MTPConfig(depth=1),
            tokenizer_slots=_small_slots(8180),
        )

    @classmethod
    def bench_1b(cls) -> ModelConfig:
        """Config 2: ~1B MoE, d 1536, 16 layers, 12x128 heads, 32 experts top-4 + 1 shared."""
        return cls(
            n_layers=16, hidden_dim=1536, vocab_size=32768, first_dense_swa_layers=0,
            attention=AttentionConfig(query_heads=12, head_dim=128, query_compression_dim=768,
                                      output_proj_groups=4, attention_intermediate_dim=768),
            moe=MoEConfig(hash_routed_layers=0, shared_experts=1, routed_experts=32,
                          experts_per_token=4, expert_intermediate_dim=1024),
            tokenizer_slots=_small_slots(32700),
            moe_use_grouped_gemm=True,
        )

    @classmethod
    def bench_16b(cls) -> ModelConfig:
        """Config 3 (headline): ~16B total / ~2.7B active FP8 MoE.

        d 2048, 28 layers, 16 heads of dim 128 (16x128 = d_model), 64 routed experts
        top-6 + 2 shared, expert hidden 1408, MTP depth 1, vocab 32768 (as configs 2
        and 4), block-scaled FP8 linears (128x128 weight / 1x128 activation blocks).
        Other attention fields keep the reference defaults (d_c 1024, g 8, d_g 1024,
        window 128, rope 64, CSA m 4 / 64x128 indexer / top-512, HCA m' 128, mHC n 4).
        """
        return cls(
            n_layers=28, hidden_dim=2048, vocab_size=32768, first_dense_swa_layers=0,
            attention=AttentionConfig(query_heads=16, head_dim=128),
            moe=MoEConfig(hash_routed_layers=0, shared_experts=2, routed_experts=64,
                          experts_per_token=6, expert_intermediate_dim=1408),
            mtp=MTPConfig(depth=1),
            tokenizer_slots=_small_slots(32700),
            linear_quant="fp8", fp8_use_real_gemm=True, moe_use_grouped_gemm=True,
        )

    @classmethod
    def bench_long(cls) -> ModelConfig:
        """Config 4: long-context CSA/HCA, d 2048, 24 layers, CSA m 128 top-16, HCA m' 16."""
        return cls(
            n_layers=24, hidden_dim=2048, vocab_size=32768, first_dense_swa_layers=0,
            csa=CSAConfig(compression_rate=128, attention_top_k=16),
            hca=HCAConfig(compression_rate=16),
            attention=AttentionConfig(query_heads=16, head_dim=128),
            moe=MoEConfig(hash_routed_layers=0, shared_experts=1, routed_experts=16,
                          experts_per_token=2, expert_intermediate_dim=1408),
            tokenizer_slots=_small_slots(32700),
            moe_use_grouped_gemm=True,
        )

    @classmethod
    def bench_decode(cls) -> ModelConfig:
        """Config 5: decode on the config-3 architecture with a 4096-token SW window."""
        base = cls.bench_16b()
        return base.model_copy(update={
            "attention": base.attention.model_copy(update={"sliding_window_size": 4096}),
        })


ParallelMode = Literal["none", "dp", "fsdp", "hybrid_zero"]


class RunConfig(_Frozen):
    """How a model runs: parallel layout, precision recipe, kernel toggles, timeouts.

    Every fused communication path has an NCCL fallback selected here, which is both
    the correctness oracle and the baseline a fused kernel is measured against.
    """

    # parallel dims (product of ep/dp must equal world size; tp/cp/pp divide it)
    ep: int = 1
    tp: int = 1
    cp: int = 1
    pp: int = 1
    zero: ParallelMode = "dp"
    # pipeline schedule with pp > 1: one-forward-one-backward, or the V-shaped DualPipe-V
    pp_schedule: Literal["1f1b", "dualpipe"] = "1f1b"
    # precision
    compute_dtype: Literal["bfloat16", "float32"] = "bfloat16"
    param_dtype: Literal["bfloat16", "float32"] = "bfloat16"
    grad_dtype: Literal["bfloat16", "float32"] = "float32"
    # kernels: "native" = our sm_100a kernels, "torch" = eager oracle path
    kernels: Literal["native", "torch"] = "native"
    fused_ep: bool = True
    fused_zero: bool = True
    # tensor parallelism (tp > 1): the attention block's output projection and input gradient
    # reduced by the NVLink peer-memory kernels (True) or NCCL all-reduces (False)
    fused_tp: bool = False
    # hybrid ZeRO transport: "nccl" (reduce / broadcast), "p2p" (owners pull gradients and
    # parameters over NVLink peer memory, parallel.zero_p2p) or "auto" (p2p on CUDA)
    zero_transport: Literal["auto", "nccl", "p2p"] = "auto"
    # single GPU: replay each micro-batch's forward + backward from one captured CUDA graph
    cuda_graphs: bool = True
    # FP8 training (linear_quant="fp8"): keep the routed experts' FP8 weight copies between
    # steps ("always"), quantise them per forward ("never"), or cache them only when expert
    # parallelism shards the pools ("auto": an unsharded 16B pool's copy does not fit)
    fp8_expert_cache: Literal["auto", "always", "never"] = "auto"
    # training loop
    micro_batch: int = 1
    seq_len: int = 4096
    grad_accum: int = 1
    lr: float = 2.7e-4
    adamw_lr: float = 2.7e-4
    # runtime
    pg_timeout_s: float = 120.0
    # bound of every cross-GPU flag wait in the peer-memory kernels (ranks may start a step
    # seconds apart, e.g. after an uneven optimizer step); a timed-out wait raises
    device_wait_timeout_ms: int = 30000
    seed: int = 0

    @classmethod
    def from_file(cls, path: str | Path) -> RunConfig:
        p = Path(path)
        text = p.read_text()
        if p.suffix in (".yaml", ".yml"):
            import yaml

            data: dict[str, Any] = yaml.safe_load(text) or {}
        else:
            data = json.loads(text)
        return cls.model_validate(data)

    def with_overrides(self, **kw: Any) -> RunConfig:
        return self.model_copy(update=kw)


__all__ = [
    "AttentionConfig",
    "CSAConfig",
    "HCAConfig",
    "NSAConfig",
    "MHCConfig",
    "MTPConfig",
    "MoEConfig",
    "ModelConfig",
    "MultimodalConfig",
    "RunConfig",
    "TokenizerSlots",
]

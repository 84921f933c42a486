"""Attention family: SWA, CSA (+ compressor, lightning indexer), HCA, NSA, tree and
deterministic attention."""

from saint_llm_b200.models.attention.common import (
    RMSNorm,
    apply_partial_rope,
    build_rope_cache,
    causal_mask,
    rope_tables,
    scaled_dot_product,
    sliding_window_mask,
    softmax_with_sink,
)
from saint_llm_b200.models.attention.csa import CSA, GroupedOutputProjection, LightningIndexer, TokenLevelCompressor
from saint_llm_b200.models.attention.swa import HCA, SWAttention

__all__ = [
    "CSA",
    "HCA",
    "GroupedOutputProjection",
    "LightningIndexer",
    "RMSNorm",
    "SWAttention",
    "TokenLevelCompressor",
    "apply_partial_rope",
    "build_rope_cache",
    "causal_mask",
    "rope_tables",
    "scaled_dot_product",
    "sliding_window_mask",
    "softmax_with_sink",
]

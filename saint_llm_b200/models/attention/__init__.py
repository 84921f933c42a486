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
from saint_llm_b200.models.attention.deterministic import batch_invariant_attention, deterministic_mode
from saint_llm_b200.models.attention.nsa import NSAttention
from saint_llm_b200.models.attention.swa import HCA, SWAttention
from saint_llm_b200.models.attention.tree import merge_partials, tree_attention, tree_attention_distributed

__all__ = [
    "CSA",
    "HCA",
    "GroupedOutputProjection",
    "LightningIndexer",
    "NSAttention",
    "RMSNorm",
    "SWAttention",
    "TokenLevelCompressor",
    "apply_partial_rope",
    "batch_invariant_attention",
    "build_rope_cache",
    "causal_mask",
    "deterministic_mode",
    "merge_partials",
    "rope_tables",
    "scaled_dot_product",
    "sliding_window_mask",
    "softmax_with_sink",
    "tree_attention",
    "tree_attention_distributed",
]

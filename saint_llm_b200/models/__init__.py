"""Model layer: the V4-style SaintLLM and its components."""

from saint_llm_b200.models.attention import CSA, HCA, RMSNorm, SWAttention
from saint_llm_b200.models.linear import Fp4Linear, Fp8Linear, Linear, make_linear_factory
from saint_llm_b200.models.mhc import MHC, sinkhorn_knopp
from saint_llm_b200.models.model import SaintLLM, TransformerBlock
from saint_llm_b200.models.moe import DeepSeekMoE, HashRouter, LearnedRouter, SwiGLU
from saint_llm_b200.models.mtp import MTPModule, MTPStack

__all__ = [
    "CSA",
    "HCA",
    "MHC",
    "DeepSeekMoE",
    "Fp4Linear",
    "Fp8Linear",
    "HashRouter",
    "LearnedRouter",
    "Linear",
    "MTPModule",
    "MTPStack",
    "RMSNorm",
    "SWAttention",
    "SaintLLM",
    "SwiGLU",
    "TransformerBlock",
    "make_linear_factory",
    "sinkhorn_knopp",
]

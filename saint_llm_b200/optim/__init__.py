"""Optimizers: Muon (hybrid Newton-Schulz, MuonClip), combined Muon/AdamW, param split."""

from saint_llm_b200.optim.muon import Muon, MuonAdamW
from saint_llm_b200.optim.newton_schulz import batched_newton_schulz, hybrid_newton_schulz
from saint_llm_b200.optim.param_groups import split_for_muon_adamw

__all__ = ["Muon", "MuonAdamW", "batched_newton_schulz", "hybrid_newton_schulz", "split_for_muon_adamw"]

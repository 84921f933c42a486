"""Evaluation: perplexity and an lm-eval-harness compatible model adapter."""

from saint_llm_b200.eval.harness import SaintLLMHarnessLM
from saint_llm_b200.eval.perplexity import compute_perplexity, compute_perplexity_streaming, token_nll

__all__ = ["SaintLLMHarnessLM", "compute_perplexity", "compute_perplexity_streaming", "token_nll"]

"""Inference: heterogeneous KV cache, decoding loops, sampling, streaming, stop
sequences, logit bias, chat sessions, multimodal decoding, speculative decoding, Engram."""

from saint_llm_b200.infer.chat import ChatSession, GenerationConfig, MultimodalChatSession
from saint_llm_b200.infer.eagle3 import EAGLE3Config, EAGLE3DraftHead, speculative_decode
from saint_llm_b200.infer.engram import EngramConfig, EngramHook, EngramTable
from saint_llm_b200.infer.generate import (
    decode,
    greedy_decode,
    greedy_decode_cached,
    top_k_sample,
    top_k_sample_cached,
    top_p_sample,
    top_p_sample_cached,
)
from saint_llm_b200.infer.kv_cache import CSAKVCacheLayer, HCAKVCacheLayer, KVCacheBundle, SWAKVCacheLayer
from saint_llm_b200.infer.logit_bias import apply_logit_bias, forbid_tokens_bias, force_token_bias
from saint_llm_b200.infer.multimodal_generate import (
    MultimodalSlots,
    build_multimodal_prompt_ids,
    multimodal_greedy_decode,
)
from saint_llm_b200.infer.sampling import SamplingParams
from saint_llm_b200.infer.stop_sequences import StopSequenceMatcher, encode_stop_strings
from saint_llm_b200.infer.streaming import stream_greedy_decode, stream_top_p_sample

__all__ = [
    "CSAKVCacheLayer", "ChatSession", "EAGLE3Config", "EAGLE3DraftHead", "EngramConfig", "EngramHook", "EngramTable",
    "GenerationConfig", "HCAKVCacheLayer", "KVCacheBundle", "MultimodalChatSession", "MultimodalSlots",
    "SWAKVCacheLayer", "SamplingParams", "StopSequenceMatcher", "apply_logit_bias", "build_multimodal_prompt_ids",
    "decode", "encode_stop_strings", "forbid_tokens_bias", "force_token_bias", "greedy_decode", "greedy_decode_cached",
    "multimodal_greedy_decode", "speculative_decode", "stream_greedy_decode", "stream_top_p_sample", "top_k_sample",
    "top_k_sample_cached", "top_p_sample", "top_p_sample_cached",
]

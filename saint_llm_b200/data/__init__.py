"""Data: tokenizers, packing, datasets, corpus mixing, BBPE training, chat rendering,
multimodal packing, fertility, the document pipeline and the native token-shard loader."""

from saint_llm_b200.data.bbpe import (
    DEFAULT_SPECIAL_TOKENS,
    SAINT_V0_0_FORCE_INCLUDE_CHARS,
    SAINT_V0_0_SPECIAL_TOKENS,
    train_bbpe,
)
from saint_llm_b200.data.chat_template import ChatTemplate, ChatTurn, RenderedChat, render_chat
from saint_llm_b200.data.datasets import HuggingFaceTextDataset, ParquetShardDataset, TextFileDataset
from saint_llm_b200.data.fertility import (
    FertilityRecord,
    FertilityReport,
    measure_fertility,
    measure_per_language_fertility,
)
from saint_llm_b200.data.mix_corpus import CorpusSlice, MixedCorpus
from saint_llm_b200.data.multimodal import (
    MultimodalExample,
    MultimodalPackedBatch,
    TokenSlots,
    encode_multimodal,
    pack_multimodal_examples,
)
from saint_llm_b200.data.multimodal_chat import (
    MultimodalChatTurn,
    RenderedMultimodalChat,
    render_multimodal_chat,
    render_text_chat_to_multimodal,
    to_chat_turn,
)
from saint_llm_b200.data.packing import PackedBatch, pack_flat, pack_into_batch, pack_sequences
from saint_llm_b200.data.token_loader import ShardedTokenLoader, read_token_shard, write_token_shard
from saint_llm_b200.data.tokenizer import CharTokenizer, HFTokenizer, Tokenizer

__all__ = [
    "DEFAULT_SPECIAL_TOKENS", "SAINT_V0_0_FORCE_INCLUDE_CHARS", "SAINT_V0_0_SPECIAL_TOKENS", "CharTokenizer",
    "ChatTemplate", "ChatTurn", "CorpusSlice", "FertilityRecord", "FertilityReport", "HFTokenizer",
    "HuggingFaceTextDataset", "MixedCorpus", "MultimodalChatTurn", "MultimodalExample", "MultimodalPackedBatch",
    "PackedBatch", "ParquetShardDataset", "RenderedChat", "RenderedMultimodalChat", "ShardedTokenLoader",
    "TextFileDataset", "TokenSlots", "Tokenizer", "encode_multimodal", "measure_fertility",
    "measure_per_language_fertility", "pack_flat", "pack_into_batch", "pack_multimodal_examples", "pack_sequences",
    "read_token_shard", "render_chat", "render_multimodal_chat", "render_text_chat_to_multimodal", "to_chat_turn",
    "train_bbpe", "write_token_shard",
]

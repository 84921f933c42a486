"""Byte-level BPE training with the project's reserved special tokens.

Recipe as in the reference (``saint_llm_data/tokenizer_trainer.py:46-200``): byte-level
pre-tokenizer/decoder, the 256-symbol byte alphabet plus forced extra seeds, BPE-dropout
during training (disabled in the saved tokenizer), special tokens at the lowest ids.  The
special-token list and its order are part of the checkpoint/tokenizer format.
"""

from __future__ import annotations

import json
from collections.abc import Iterable
from pathlib import Path

from saint_llm_b200.data.tokenizer import HFTokenizer

DEFAULT_SPECIAL_TOKENS: tuple[str, ...] = (
    "<pad>", "<|endoftext|>", "<|bos|>", "<unk>", "<|image_pad|>", "<|audio_start|>", "<|audio_end|>",
    "<|video_start|>", "<|video_end|>", "<|think_start|>", "<|think_end|>",
)

SAINT_V0_0_SPECIAL_TOKENS: tuple[str, ...] = (
    *DEFAULT_SPECIAL_TOKENS[:9], "<|think_start|>", "<|think_end|>", "<|reflect|>", "</reflect|>",
    *(f"<|effort:{i}|>" for i in range(5)),
    "<|memory_recall|>", "<|memory_save|>", "<|memory_result|>",
    "<|action|>", "<|title|>", "<|query|>",
)

# Ukrainian letters and apostrophe variants seeded as whole symbols.
SAINT_V0_0_FORCE_INCLUDE_CHARS: tuple[str, ...] = (
    "ї", "Ї", "є", "Є", "ґ", "Ґ", "і", "І", "'", "ʼ", "’",
)


def train_bbpe(corpus: Iterable[str], output_path: str | Path, *, vocab_size: int = 32_000, min_frequency: int = 2,
               dropout: float | None = 0.1, special_tokens: Iterable[str] = DEFAULT_SPECIAL_TOKENS,
               force_include_chars: Iterable[str] = (), show_progress: bool = False,
               eos_token: str = "<|endoftext|>", pad_token: str = "<pad>") -> HFTokenizer:
    from tokenizers import Tokenizer as _Backend
    from tokenizers import decoders, models, pre_tokenizers, processors, trainers

    out = Path(output_path)
    out.parent.mkdir(parents=True, exist_ok=True)
    tok = _Backend(models.BPE(unk_token="<unk>", dropout=dropout))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    tok.post_processor = processors.ByteLevel(trim_offsets=True)
    alphabet = list(pre_tokenizers.ByteLevel.alphabet())
    alphabet += [c for c in dict.fromkeys(force_include_chars) if c not in alphabet]
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, min_frequency=min_frequency,
                                  special_tokens=list(special_tokens), initial_alphabet=alphabet,
                                  show_progress=show_progress)
    tok.train_from_iterator(corpus, trainer=trainer)
    if dropout is not None:
        # Inference tokenizers are deterministic: rebuild the model without dropout.
        state = json.loads(tok.to_str())
        state["model"]["dropout"] = None
        tok = _Backend.from_str(json.dumps(state))
    tok.save(str(out))
    return HFTokenizer.from_file(out, eos_token=eos_token, pad_token=pad_token)


__all__ = ["DEFAULT_SPECIAL_TOKENS", "SAINT_V0_0_FORCE_INCLUDE_CHARS", "SAINT_V0_0_SPECIAL_TOKENS", "train_bbpe"]

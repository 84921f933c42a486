"""Multimodal examples -> packed windows with placeholder slots and aligned features.

Token layout per example (reference format, ``saint_llm_data/multimodal.py:39-270``):
``prompt, <|image_pad|> x patches per image, [<|audio_start|>, <|audio_start|> x n,
<|audio_end|>] per clip, response, eos``; loss only on response + eos.

Features are kept aligned with the slots the model fills: the model splices one vision
row per ``<|image_pad|>`` and one audio row per token in ``[audio_start, audio_end]``
(the two bracket tokens included, which get zero rows).  Unlike a per-window dump of
whole examples' features, a window here carries exactly the feature rows of the slots
inside it, so an example split across windows stays consistent with the model.
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator
from dataclasses import dataclass

import torch
from torch import Tensor

from saint_llm_b200.data.tokenizer import Tokenizer


@dataclass(frozen=True)
class MultimodalExample:
    prompt: str
    response: str
    image_features: tuple[Tensor, ...] = ()
    audio_features: tuple[Tensor, ...] = ()


@dataclass(frozen=True)
class MultimodalPackedBatch:
    tokens: Tensor
    loss_mask: Tensor
    segment_ids: Tensor
    vision_features: Tensor | None = None
    audio_features: Tensor | None = None


@dataclass(frozen=True)
class TokenSlots:
    image_pad: int
    audio_start: int
    audio_end: int

    @classmethod
    def from_tokenizer(cls, tokenizer: Tokenizer, *, image_pad: str = "<|image_pad|>",
                       audio_start: str = "<|audio_start|>", audio_end: str = "<|audio_end|>") -> TokenSlots:
        lookup = getattr(tokenizer, "token_to_id", None)
        if lookup is None:
            raise ValueError(f"{type(tokenizer).__name__} cannot look up special tokens")
        ids = {n: lookup(t) for n, t in (("image_pad", image_pad), ("audio_start", audio_start),
                                         ("audio_end", audio_end))}
        missing = [n for n, v in ids.items() if v is None]
        if missing:
            raise ValueError(f"tokenizer is missing special tokens: {missing}")
        return cls(**{k: int(v) for k, v in ids.items()})

    @classmethod
    def from_model_config(cls, cfg: object) -> TokenSlots:
        s = cfg.tokenizer_slots  # type: ignore[attr-defined]
        return cls(image_pad=s.image_pad, audio_start=s.audio_start, audio_end=s.audio_end)


def audio_slot_rows(clip: Tensor) -> Tensor:
    """Feature rows for one clip's slots: zero row, the clip, zero row."""
    z = clip.new_zeros(1, clip.shape[1])
    return torch.cat([z, clip, z])


def encode_multimodal(example: MultimodalExample, tokenizer: Tokenizer, slots: TokenSlots, *,
                      append_eos: bool = True) -> tuple[list[int], list[int]]:
    ids = tokenizer.encode(example.prompt)
    mask = [0] * len(ids)
    for img in example.image_features:
        ids += [slots.image_pad] * int(img.shape[0])
    for clip in example.audio_features:
        ids += [slots.audio_start] * (int(clip.shape[0]) + 1) + [slots.audio_end]
    mask += [0] * (len(ids) - len(mask))
    resp = tokenizer.encode(example.response) + ([tokenizer.eos_token_id] if append_eos else [])
    return ids + resp, mask + [1] * len(resp)


def pack_multimodal_examples(examples: Iterable[MultimodalExample], tokenizer: Tokenizer, slots: TokenSlots, *,
                             seq_len: int, pad_token_id: int = 0, append_eos: bool = True,
                             drop_last: bool = True) -> Iterator[MultimodalPackedBatch]:
    if seq_len <= 0:
        raise ValueError(f"seq_len must be positive; got {seq_len}")
    toks: list[int] = []
    mask: list[int] = []
    segs: list[int] = []
    vis: list[Tensor] = []   # one row per image slot still in the buffer
    aud: list[Tensor] = []   # one row per audio slot still in the buffer
    seg = 0

    def take_rows(rows: list[Tensor], n: int) -> tuple[Tensor | None, list[Tensor]]:
        if n == 0:
            return None, rows
        flat = torch.cat(rows)
        return flat[:n], ([flat[n:]] if flat.shape[0] > n else [])

    def emit() -> MultimodalPackedBatch:
        nonlocal toks, mask, segs, vis, aud
        w = toks[:seq_len]
        n_img = sum(1 for t in w if t == slots.image_pad)
        n_aud = sum(1 for t in w if slots.audio_start <= t <= slots.audio_end)
        v, vis = take_rows(vis, n_img)
        a, aud = take_rows(aud, n_aud)
        out = MultimodalPackedBatch(torch.tensor([w]), torch.tensor([mask[:seq_len]]),
                                    torch.tensor([segs[:seq_len]]), v, a)
        toks, mask, segs = toks[seq_len:], mask[seq_len:], segs[seq_len:]
        return out

    for ex in examples:
        ids, m = encode_multimodal(ex, tokenizer, slots, append_eos=append_eos)
        if not ids:
            continue
        toks += ids
        mask += m
        segs += [seg] * len(ids)
        vis += list(ex.image_features)
        aud += [audio_slot_rows(c) for c in ex.audio_features]
        seg += 1
        while len(toks) >= seq_len:
            yield emit()
    if toks and not drop_last:
        k = seq_len - len(toks)
        toks, mask, segs = toks + [pad_token_id] * k, mask + [0] * k, segs + [segs[-1]] * k
        yield emit()


__all__ = ["MultimodalExample", "MultimodalPackedBatch", "TokenSlots", "audio_slot_rows", "encode_multimodal",
           "pack_multimodal_examples"]

"""Supervised fine-tuning: response-masked next-token CE over packed examples
(reference: ``saint_llm_posttraining/sft.py:38-233``, ``sft_dataset.py``,
``multimodal_sft.py``).  On CUDA the loss runs on the fused LM-head CE kernel with
per-token weights (the mask), so the (B, T, V) logits are never materialised."""

from __future__ import annotations

import json
from collections.abc import Iterable, Iterator
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.data import IterableDataset, get_worker_info

from saint_llm_b200.data.multimodal import MultimodalPackedBatch
from saint_llm_b200.data.tokenizer import Tokenizer


@dataclass(frozen=True)
class SFTExample:
    prompt: str
    response: str
    system: str | None = None


@dataclass(frozen=True)
class SFTPackedBatch:
    tokens: Tensor
    loss_mask: Tensor
    segment_ids: Tensor

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.tokens.shape)


def encode_sft(example: SFTExample, tokenizer: Tokenizer, *, append_eos: bool = True) -> tuple[list[int], list[int]]:
    prefix = tokenizer.encode((example.system + "\n" if example.system else "") + example.prompt)
    resp = tokenizer.encode(example.response) + ([tokenizer.eos_token_id] if append_eos else [])
    return prefix + resp, [0] * len(prefix) + [1] * len(resp)


def pack_sft_examples(examples: Iterable[SFTExample], tokenizer: Tokenizer, *, seq_len: int, pad_token_id: int = 0,
                      append_eos: bool = True, drop_last: bool = True) -> Iterator[SFTPackedBatch]:
    if seq_len <= 0:
        raise ValueError(f"seq_len must be positive; got {seq_len}")
    tok: list[int] = []
    msk: list[int] = []
    seg: list[int] = []
    n = 0
    for ex in examples:
        ids, m = encode_sft(ex, tokenizer, append_eos=append_eos)
        if not ids:
            continue
        tok += ids
        msk += m
        seg += [n] * len(ids)
        n += 1
        while len(tok) >= seq_len:
            yield SFTPackedBatch(torch.tensor([tok[:seq_len]]), torch.tensor([msk[:seq_len]]),
                                 torch.tensor([seg[:seq_len]]))
            tok, msk, seg = tok[seq_len:], msk[seq_len:], seg[seq_len:]
    if tok and not drop_last:
        k = seq_len - len(tok)
        yield SFTPackedBatch(torch.tensor([tok + [pad_token_id] * k]), torch.tensor([msk + [0] * k]),
                             torch.tensor([seg + [seg[-1]] * k]))


def pack_sft_into_batch(examples: Iterable[SFTExample], tokenizer: Tokenizer, *, batch_size: int, seq_len: int,
                        pad_token_id: int = 0, append_eos: bool = True, drop_last: bool = True
                        ) -> Iterator[SFTPackedBatch]:
    rows: list[SFTPackedBatch] = []

    def cat(rs: list[SFTPackedBatch], pad_rows: int) -> SFTPackedBatch:
        t = [r.tokens for r in rs] + [torch.full((pad_rows, seq_len), pad_token_id)] * bool(pad_rows)
        m = [r.loss_mask for r in rs] + [torch.zeros(pad_rows, seq_len, dtype=torch.long)] * bool(pad_rows)
        s = [r.segment_ids for r in rs] + [torch.full((pad_rows, seq_len), -1)] * bool(pad_rows)
        return SFTPackedBatch(torch.cat(t), torch.cat(m), torch.cat(s))

    for w in pack_sft_examples(examples, tokenizer, seq_len=seq_len, pad_token_id=pad_token_id,
                               append_eos=append_eos, drop_last=drop_last):
        rows.append(w)
        if len(rows) == batch_size:
            yield cat(rows, 0)
            rows = []
    if rows and not drop_last:
        yield cat(rows, batch_size - len(rows))


def masked_next_token_ce(logits: Tensor, tokens: Tensor, loss_mask: Tensor) -> tuple[Tensor, int]:
    """Mean CE of position t predicting t+1 over positions whose target has mask 1."""
    mask = loss_mask[:, 1:].to(device=logits.device, dtype=torch.float32)
    ce = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(),
                         tokens[:, 1:].reshape(-1).to(logits.device), reduction="none").view_as(mask)
    return (ce * mask).sum() / mask.sum().clamp(min=1.0), int(mask.sum())


def sft_cross_entropy(out: dict, batch: SFTPackedBatch) -> Tensor:
    logits = out["logits"]
    if not isinstance(logits, Tensor):
        raise TypeError("out['logits'] must be a Tensor")
    return masked_next_token_ce(logits, batch.tokens, batch.loss_mask)[0]


def sft_loss(model: nn.Module, tokens: Tensor, loss_mask: Tensor, *, vision_features: Tensor | None = None,
             audio_features: Tensor | None = None) -> Tensor:
    """Response-masked CE straight from the model (fused LM-head kernel on CUDA)."""
    from saint_llm_b200.posttrain.grpo import policy_token_logprobs

    lp = policy_token_logprobs(model, tokens, vision_features=vision_features, audio_features=audio_features)
    mask = loss_mask[:, 1:].to(lp.device, torch.float32)
    return -(lp[:, 1:] * mask).sum() / mask.sum().clamp(min=1.0)


def _iter_jsonl_examples(path: Path, *, prompt_field: str, response_field: str,
                         system_field: str | None) -> Iterator[SFTExample]:
    with path.open("r", encoding="utf-8") as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                obj = json.loads(line)
            except json.JSONDecodeError:
                continue
            p, r = obj.get(prompt_field), obj.get(response_field)
            if not isinstance(p, str) or not isinstance(r, str):
                continue
            s = obj.get(system_field) if system_field else None
            yield SFTExample(p, r, s if isinstance(s, str) else None)


class JsonlSFTDataset(IterableDataset):
    """JSONL rows ``{prompt, response[, system]}`` -> packed SFT batches (lines split across workers)."""

    def __init__(self, path: str | Path, *, tokenizer: Tokenizer, seq_len: int, batch_size: int = 1,
                 prompt_field: str = "prompt", response_field: str = "response", system_field: str | None = "system",
                 append_eos: bool = True, drop_last: bool = True) -> None:
        super().__init__()
        self.path = Path(path)
        if not self.path.exists():
            raise FileNotFoundError(f"SFT JSONL file not found: {self.path}")
        self.tokenizer, self.seq_len, self.batch_size = tokenizer, seq_len, batch_size
        self.fields = (prompt_field, response_field, system_field)
        self.append_eos, self.drop_last = append_eos, drop_last

    def _examples(self) -> Iterator[SFTExample]:
        info = get_worker_info()
        wid, nw = (0, 1) if info is None else (info.id, info.num_workers)
        for i, ex in enumerate(_iter_jsonl_examples(self.path, prompt_field=self.fields[0],
                                                    response_field=self.fields[1], system_field=self.fields[2])):
            if i % nw == wid:
                yield ex

    def __iter__(self) -> Iterator[SFTPackedBatch]:
        return pack_sft_into_batch(self._examples(), self.tokenizer, batch_size=self.batch_size, seq_len=self.seq_len,
                                   append_eos=self.append_eos, drop_last=self.drop_last)


@dataclass
class MultimodalSFTOutput:
    loss: Tensor
    n_response_tokens: int
    logits_for_aux: Tensor | None


def multimodal_sft_loss(logits: Tensor, batch: MultimodalPackedBatch) -> tuple[Tensor, int]:
    return masked_next_token_ce(logits, batch.tokens, batch.loss_mask)


def multimodal_sft_step(model: nn.Module, batch: MultimodalPackedBatch) -> MultimodalSFTOutput:
    """Forward with the window's features spliced in; returns the masked CE (no optimizer step)."""
    dev = next(model.parameters()).device
    feats = {"vision_features": None if batch.vision_features is None else batch.vision_features.to(dev),
             "audio_features": None if batch.audio_features is None else batch.audio_features.to(dev)}
    out = model(batch.tokens.to(dev), **feats)
    loss, n = multimodal_sft_loss(out["logits"], batch)
    return MultimodalSFTOutput(loss, n, out["logits"])


__all__ = ["JsonlSFTDataset", "MultimodalSFTOutput", "SFTExample", "SFTPackedBatch", "encode_sft",
           "masked_next_token_ce", "multimodal_sft_loss", "multimodal_sft_step", "pack_sft_examples",
           "pack_sft_into_batch", "sft_cross_entropy", "sft_loss"]

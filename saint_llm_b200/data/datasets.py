"""Streaming text datasets -> packed batches: plain/JSONL files, HF ``datasets`` and
parquet shards of pre-tokenised ids.  Each is an ``IterableDataset`` that splits its
documents across DataLoader workers round-robin (reference behaviour,
``saint_llm_data/dataset.py:59``, ``hf_dataset.py:30``, ``parquet_shards.py:30``).
"""

from __future__ import annotations

import json
from collections.abc import Iterable, Iterator
from pathlib import Path
from typing import Any

from torch.utils.data import IterableDataset, get_worker_info

from saint_llm_b200.data.packing import PackedBatch, pack_into_batch
from saint_llm_b200.data.tokenizer import Tokenizer


def worker_shard() -> tuple[int, int]:
    info = get_worker_info()
    return (0, 1) if info is None else (int(info.id), int(info.num_workers))


def iter_text_lines(path: Path, *, jsonl: bool, json_field: str) -> Iterator[str]:
    with path.open("r", encoding="utf-8") as f:
        for line in f:
            line = line.rstrip("\n")
            if not line:
                continue
            if not jsonl:
                yield line
                continue
            obj = json.loads(line)
            if json_field not in obj:
                raise KeyError(f"JSONL record in {path.name} has no field {json_field!r} (keys: {sorted(obj)})")
            yield str(obj[json_field])


class _PackedTextDataset(IterableDataset):
    def __init__(self, tokenizer: Tokenizer, seq_len: int, batch_size: int, drop_last: bool) -> None:
        super().__init__()
        self.tokenizer, self.seq_len, self.batch_size, self.drop_last = tokenizer, seq_len, batch_size, drop_last

    def _docs(self) -> Iterable[list[int]]:
        raise NotImplementedError

    def __iter__(self) -> Iterator[PackedBatch]:
        return pack_into_batch(self._docs(), batch_size=self.batch_size, seq_len=self.seq_len,
                               eos_token_id=self.tokenizer.eos_token_id, pad_token_id=self.tokenizer.pad_token_id,
                               drop_last=self.drop_last)


class TextFileDataset(_PackedTextDataset):
    """One document per line (or per JSONL record's ``json_field``)."""

    def __init__(self, path: str | Path, tokenizer: Tokenizer, *, seq_len: int, batch_size: int = 1,
                 jsonl: bool = False, json_field: str = "text", drop_last: bool = True) -> None:
        super().__init__(tokenizer, seq_len, batch_size, drop_last)
        self.path = Path(path)
        if not self.path.exists():
            raise FileNotFoundError(self.path)
        self.jsonl, self.json_field = jsonl, json_field

    def _docs(self) -> Iterable[list[int]]:
        wid, nw = worker_shard()
        for i, text in enumerate(iter_text_lines(self.path, jsonl=self.jsonl, json_field=self.json_field)):
            if i % nw == wid:
                yield self.tokenizer.encode(text)


class HuggingFaceTextDataset(_PackedTextDataset):
    """Rows of a ``datasets`` dataset (streaming by default); ``text_field`` holds the text."""

    def __init__(self, path: str, tokenizer: Tokenizer, *, seq_len: int, batch_size: int = 1, split: str = "train",
                 text_field: str = "text", streaming: bool = True, config: str | None = None,
                 drop_last: bool = True, load_dataset_kwargs: dict[str, Any] | None = None) -> None:
        super().__init__(tokenizer, seq_len, batch_size, drop_last)
        self.path, self.split, self.text_field = path, split, text_field
        self.streaming, self.config = streaming, config
        self.load_dataset_kwargs = dict(load_dataset_kwargs or {})

    def _open(self) -> Iterable[dict[str, Any]]:
        from datasets import load_dataset  # optional dependency

        args = (self.path,) if self.config is None else (self.path, self.config)
        return load_dataset(*args, split=self.split, streaming=self.streaming, **self.load_dataset_kwargs)

    def _docs(self) -> Iterable[list[int]]:
        wid, nw = worker_shard()
        for i, row in enumerate(self._open()):
            if i % nw != wid:
                continue
            if self.text_field not in row:
                raise KeyError(f"row has no field {self.text_field!r} (keys: {sorted(row)})")
            text = row[self.text_field]
            if not isinstance(text, str):
                raise TypeError(f"field {self.text_field!r} is {type(text).__name__}, not str")
            if text:
                yield self.tokenizer.encode(text)


class ParquetShardDataset(_PackedTextDataset):
    """Parquet files with a ``token_ids`` list column; shards are split across workers."""

    def __init__(self, shard_dir: str | Path, *, tokenizer: Tokenizer, seq_len: int, batch_size: int = 1,
                 drop_last: bool = True, shard_glob: str = "*.parquet") -> None:
        super().__init__(tokenizer, seq_len, batch_size, drop_last)
        self.shard_dir = Path(shard_dir)
        if not self.shard_dir.exists():
            raise FileNotFoundError(f"shard_dir not found: {self.shard_dir}")
        self.shard_glob = shard_glob

    def shards(self) -> list[Path]:
        wid, nw = worker_shard()
        return [s for i, s in enumerate(sorted(self.shard_dir.glob(self.shard_glob))) if i % nw == wid]

    def _docs(self) -> Iterable[list[int]]:
        import pyarrow.parquet as pq

        for shard in self.shards():
            for batch in pq.ParquetFile(str(shard)).iter_batches(columns=["token_ids"]):
                for ids in batch.column(0).to_pylist():
                    if ids:
                        yield list(ids)


__all__ = ["HuggingFaceTextDataset", "ParquetShardDataset", "TextFileDataset", "iter_text_lines", "worker_shard"]

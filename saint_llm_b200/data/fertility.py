"""Tokenizer fertility (tokens per character) per language
(reference: ``saint_llm_data/fertility.py:29-120``)."""

from __future__ import annotations

from collections.abc import Iterable, Mapping
from dataclasses import asdict, dataclass

from saint_llm_b200.data.tokenizer import Tokenizer


@dataclass(frozen=True)
class FertilityRecord:
    language: str
    n_samples: int
    chars: int
    tokens: int
    fertility: float


@dataclass(frozen=True)
class FertilityReport:
    records: tuple[FertilityRecord, ...]

    def to_dict(self) -> dict[str, object]:
        return {"records": [asdict(r) for r in self.records]}

    def by_language(self) -> dict[str, FertilityRecord]:
        return {r.language: r for r in self.records}


def measure_fertility(tokenizer: Tokenizer, text: str) -> tuple[int, int]:
    return (len(text), len(tokenizer.encode(text))) if text else (0, 0)


def measure_per_language_fertility(tokenizer: Tokenizer, samples: Mapping[str, Iterable[str]]) -> FertilityReport:
    recs = []
    for lang, texts in samples.items():
        n = chars = toks = 0
        for t in texts:
            c, k = measure_fertility(tokenizer, t)
            n, chars, toks = n + 1, chars + c, toks + k
        if chars:
            recs.append(FertilityRecord(lang, n, chars, toks, toks / chars))
    return FertilityReport(tuple(sorted(recs, key=lambda r: r.language)))


__all__ = ["FertilityRecord", "FertilityReport", "measure_fertility", "measure_per_language_fertility"]

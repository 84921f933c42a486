"""Weighted interleaving of document sources (reference: ``saint_llm_data/mix_corpus.py:29-110``).

A slice is picked with probability proportional to its weight among the slices that are
not exhausted; an exhausted slice drops out and the rest are renormalised.  Iteration
ends at ``max_docs`` or when every slice is exhausted.
"""

from __future__ import annotations

import bisect
import itertools
import random
from collections.abc import Iterable, Iterator
from dataclasses import dataclass


@dataclass(frozen=True)
class CorpusSlice:
    name: str
    weight: float
    source: Iterable[str]


class MixedCorpus:
    def __init__(self, slices: list[CorpusSlice], *, max_docs: int | None = None, seed: int = 0) -> None:
        if not slices:
            raise ValueError("MixedCorpus requires at least one slice")
        bad = [s.name for s in slices if s.weight <= 0]
        if bad:
            raise ValueError(f"slices with non-positive weight: {bad}")
        self._slices = list(slices)
        self._max_docs = max_docs
        self._rng = random.Random(seed)
        self.counts: dict[str, int] = {s.name: 0 for s in slices}

    def __iter__(self) -> Iterator[str]:
        live = [(s.name, s.weight, iter(s.source)) for s in self._slices]
        emitted = 0
        while live and (self._max_docs is None or emitted < self._max_docs):
            cum = list(itertools.accumulate(w for _, w, _ in live))
            i = min(bisect.bisect_left(cum, self._rng.uniform(0.0, cum[-1])), len(live) - 1)
            name, _, it = live[i]
            try:
                doc = next(it)
            except StopIteration:
                del live[i]
                continue
            self.counts[name] += 1
            emitted += 1
            yield doc


__all__ = ["CorpusSlice", "MixedCorpus"]

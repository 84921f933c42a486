"""Stop-sequence matching on the tail of generated tokens (reference:
``saint_llm_inference/stop_sequences.py:27-107``).  Once matched, a matcher stays matched."""

from __future__ import annotations

from collections import deque
from collections.abc import Sequence

from saint_llm_b200.data.tokenizer import Tokenizer


class StopSequenceMatcher:
    def __init__(self, sequences: Sequence[Sequence[int]]) -> None:
        self._sequences = tuple(t for t in (tuple(int(x) for x in s) for s in sequences) if t)
        self._max = max(map(len, self._sequences), default=0)
        self._tail: deque[int] = deque(maxlen=max(self._max, 1))
        self._hit: tuple[int, ...] | None = None

    @property
    def sequences(self) -> tuple[tuple[int, ...], ...]:
        return self._sequences

    @property
    def matched_sequence(self) -> tuple[int, ...] | None:
        return self._hit

    def feed(self, token: int) -> bool:
        if self._max == 0:
            return False
        if self._hit is not None:
            return True
        self._tail.append(int(token))
        tail = tuple(self._tail)
        for s in self._sequences:
            if tail[len(tail) - len(s):] == s and len(tail) >= len(s):
                self._hit = s
                return True
        return False

    def matched(self) -> bool:
        return self._hit is not None

    def reset(self) -> None:
        self._tail.clear()
        self._hit = None


def encode_stop_strings(stops: Sequence[str], tokenizer: Tokenizer) -> list[list[int]]:
    return [ids for ids in (list(tokenizer.encode(s)) for s in stops if s) if ids]


__all__ = ["StopSequenceMatcher", "encode_stop_strings"]

"""Tokenizers: the ``Tokenizer`` protocol, a hermetic code-point tokenizer and a wrapper
around the HF ``tokenizers`` library.

Behaviour follows the reference's ``saint_llm_data/tokenizer.py:25-160``: the code-point
tokenizer reserves ``base_vocab`` control ids (0 pad, 1 eos, 2 bos) and maps a character
to ``base_vocab + ord(ch)``; decode drops control ids.  These id layouts are part of the
interface (checkpoints trained with them must decode the same way).
"""

from __future__ import annotations

from collections.abc import Iterable
from pathlib import Path
from typing import Protocol, runtime_checkable


@runtime_checkable
class Tokenizer(Protocol):
    @property
    def vocab_size(self) -> int: ...

    @property
    def eos_token_id(self) -> int: ...

    @property
    def pad_token_id(self) -> int: ...

    def encode(self, text: str) -> list[int]: ...

    def encode_batch(self, texts: Iterable[str]) -> list[list[int]]: ...

    def decode(self, ids: Iterable[int]) -> str: ...


class CharTokenizer:
    """Unicode code point ``c`` -> id ``base_vocab + c``; ids below ``base_vocab`` are control slots."""

    PAD, EOS, BOS = 0, 1, 2

    def __init__(self, *, base_vocab: int = 16, unicode_max: int = 0x110000) -> None:
        if base_vocab < 3:
            raise ValueError("base_vocab must leave room for pad/eos/bos")
        self._base = base_vocab
        self._umax = unicode_max

    @property
    def vocab_size(self) -> int:
        return self._base + self._umax

    @property
    def pad_token_id(self) -> int:
        return self.PAD

    @property
    def eos_token_id(self) -> int:
        return self.EOS

    @property
    def bos_token_id(self) -> int:
        return self.BOS

    def encode(self, text: str) -> list[int]:
        base = self._base
        return [base + ord(c) for c in text]

    def encode_batch(self, texts: Iterable[str]) -> list[list[int]]:
        return [self.encode(t) for t in texts]

    def decode(self, ids: Iterable[int]) -> str:
        base, umax = self._base, self._umax
        return "".join(chr(i - base) for i in map(int, ids) if base <= i and i - base <= umax and i - base < 0x110000)

    def token_to_id(self, token: str) -> int | None:
        """Single-character tokens only (there are no named specials)."""
        return self._base + ord(token) if len(token) == 1 else None


class HFTokenizer:
    """Adapter over ``tokenizers.Tokenizer``; special ids are looked up by name."""

    def __init__(self, backend: object, *, eos_token: str = "<|endoftext|>", pad_token: str | None = None) -> None:
        self._backend = backend
        eos = backend.token_to_id(eos_token)  # type: ignore[attr-defined]
        if eos is None:
            raise ValueError(f"eos token {eos_token!r} is not in the tokenizer's vocabulary")
        self._eos = int(eos)
        pad = backend.token_to_id(pad_token) if pad_token else None  # type: ignore[attr-defined]
        self._pad = int(pad) if pad is not None else self._eos

    @property
    def backend(self) -> object:
        return self._backend

    @property
    def vocab_size(self) -> int:
        return int(self._backend.get_vocab_size())  # type: ignore[attr-defined]

    @property
    def eos_token_id(self) -> int:
        return self._eos

    @property
    def pad_token_id(self) -> int:
        return self._pad

    def token_to_id(self, token: str) -> int | None:
        tid = self._backend.token_to_id(token)  # type: ignore[attr-defined]
        return None if tid is None else int(tid)

    def encode(self, text: str) -> list[int]:
        return list(self._backend.encode(text).ids)  # type: ignore[attr-defined]

    def encode_batch(self, texts: Iterable[str]) -> list[list[int]]:
        return [list(e.ids) for e in self._backend.encode_batch(list(texts))]  # type: ignore[attr-defined]

    def decode(self, ids: Iterable[int]) -> str:
        return str(self._backend.decode(list(ids)))  # type: ignore[attr-defined]

    @classmethod
    def from_file(cls, path: str | Path, **kwargs: object) -> HFTokenizer:
        from tokenizers import Tokenizer as _Backend

        return cls(_Backend.from_file(str(path)), **kwargs)  # type: ignore[arg-type]

    @classmethod
    def from_pretrained(cls, identifier: str, **kwargs: object) -> HFTokenizer:
        from tokenizers import Tokenizer as _Backend

        return cls(_Backend.from_pretrained(identifier), **kwargs)  # type: ignore[arg-type]


def special_token_id(tokenizer: object, token: str) -> int | None:
    """Id of a named special token, for any tokenizer exposing ``token_to_id``."""
    fn = getattr(tokenizer, "token_to_id", None)
    return fn(token) if fn is not None else None

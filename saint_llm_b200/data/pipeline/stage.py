"""Stage protocol, the streaming ``Pipeline`` and the tokenize stage."""

from __future__ import annotations

from collections.abc import Iterable, Iterator
from dataclasses import dataclass
from typing import Any, Protocol

from saint_llm_b200.data.tokenizer import Tokenizer

Document = dict[str, Any]


class Stage(Protocol):
    name: str

    def __call__(self, doc: Document) -> Document | None: ...


@dataclass
class Pipeline:
    stages: list[Stage]

    def _through(self, doc: Document, drops: dict[str, int] | None) -> Document | None:
        cur: Document | None = doc
        for st in self.stages:
            cur = st(cur)
            if cur is None:
                if drops is not None:
                    drops[st.name] += 1
                return None
        return cur

    def run(self, source: Iterable[Document]) -> Iterator[Document]:
        for doc in source:
            out = self._through(doc, None)
            if out is not None:
                yield out

    def stats_run(self, source: Iterable[Document]) -> tuple[list[Document], dict[str, int]]:
        drops = {st.name: 0 for st in self.stages}
        kept = [d for d in (self._through(doc, drops) for doc in source) if d is not None]
        return kept, drops


@dataclass
class TokenizeStage:
    tokenizer: Tokenizer
    name: str = "tokenize"

    def __call__(self, doc: Document) -> Document | None:
        text = doc.get("text", "")
        ids = self.tokenizer.encode(text) if text else []
        if not ids:
            return None
        doc["token_ids"] = ids
        return doc

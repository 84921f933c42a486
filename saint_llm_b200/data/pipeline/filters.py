"""Quality / length / machine-translation-pollution filters
(reference: ``saint_llm_data/pipeline/quality.py:27-86``, ``mt_pollution.py:29-144``)."""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Protocol
from urllib.parse import urlparse

from saint_llm_b200.data.pipeline.stage import Document

DEFAULT_BLOCKED_DOMAINS: tuple[str, ...] = ("translated-articles.example", "auto-translate.example")


class QualityClassifier(Protocol):
    def __call__(self, text: str, *, language: str | None = None) -> float: ...


class TranslationeseDetector(Protocol):
    def __call__(self, text: str) -> float: ...


class PerplexityModel(Protocol):
    def perplexity(self, text: str) -> float: ...


def _in_scope(doc: Document, languages: tuple[str, ...]) -> bool:
    return not languages or doc.get("language") in languages


@dataclass
class QualityFilter:
    classifier: QualityClassifier
    threshold: float
    apply_to_slices: tuple[str, ...] = ()
    name: str = "quality_filter"

    def __call__(self, doc: Document) -> Document | None:
        if self.apply_to_slices and doc.get("slice", "") not in self.apply_to_slices:
            return doc
        text = doc.get("text", "")
        if not text or self.classifier(text, language=doc.get("language")) < self.threshold:
            return None
        return doc


@dataclass
class LengthQualityFilter:
    min_chars: int = 100
    min_chars_per_language: dict[str, int] | None = None
    name: str = "length_quality_filter"

    def __call__(self, doc: Document) -> Document | None:
        lim = (self.min_chars_per_language or {}).get(doc.get("language", ""), self.min_chars)
        return doc if len(doc.get("text", "")) >= lim else None


@dataclass
class URLBlocklistFilter:
    blocked_domains: tuple[str, ...] = DEFAULT_BLOCKED_DOMAINS
    apply_to_languages: tuple[str, ...] = ("uk",)
    name: str = "url_blocklist"
    _pattern: re.Pattern[str] | None = field(init=False, repr=False, default=None)

    def __post_init__(self) -> None:
        if self.blocked_domains:
            self._pattern = re.compile("|".join(re.escape(d) for d in self.blocked_domains), re.IGNORECASE)

    def __call__(self, doc: Document) -> Document | None:
        if not _in_scope(doc, self.apply_to_languages) or self._pattern is None:
            return doc
        meta = doc.get("meta", {})
        url = meta.get("url", "") if isinstance(meta, dict) else ""
        try:
            host = urlparse(url).hostname or "" if url else ""
        except ValueError:
            host = ""
        return None if host and self._pattern.search(host) else doc


@dataclass
class TranslationeseFilter:
    detector: TranslationeseDetector
    threshold: float
    apply_to_languages: tuple[str, ...] = ("uk",)
    name: str = "translationese_filter"

    def __call__(self, doc: Document) -> Document | None:
        text = doc.get("text", "")
        if not _in_scope(doc, self.apply_to_languages) or not text:
            return doc
        return None if self.detector(text) >= self.threshold else doc


@dataclass
class PerplexityFilter:
    model: PerplexityModel
    max_perplexity: float
    apply_to_languages: tuple[str, ...] = ("uk",)
    name: str = "perplexity_filter"

    def __call__(self, doc: Document) -> Document | None:
        text = doc.get("text", "")
        if not _in_scope(doc, self.apply_to_languages) or not text:
            return doc
        return None if self.model.perplexity(text) > self.max_perplexity else doc

"""Agent memory: a key -> text store (in memory, or one ``<key>.md`` file plus a ``<key>.meta``
timestamp per entry on disk) and the four memory tools (view / store / recall / delete)
(reference: ``saint_llm_agents/memory/*.py``)."""

from __future__ import annotations

import json
import re
import time
from abc import ABC, abstractmethod
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from saint_llm_b200.agents.core import FunctionTool, Tool, ToolRegistry, ToolSpec

KEY_PATTERN = re.compile(r"^[A-Za-z0-9._-]+$")


def _check_key(key: str) -> None:
    if not key or not KEY_PATTERN.match(key) or key in (".", ".."):
        raise ValueError(f"invalid memory key {key!r}: use letters, digits, '.', '_', '-'")


@dataclass(frozen=True)
class MemoryEntry:
    key: str
    value: str
    created_at: float


class MemoryStore(ABC):
    @abstractmethod
    def store(self, key: str, value: str) -> MemoryEntry: ...

    @abstractmethod
    def view(self, key: str) -> MemoryEntry | None: ...

    @abstractmethod
    def list(self) -> tuple[MemoryEntry, ...]: ...

    @abstractmethod
    def delete(self, key: str) -> bool: ...

    @abstractmethod
    def clear(self) -> None: ...

    def recall(self, query: str, *, limit: int = 5) -> tuple[MemoryEntry, ...]:
        """Case-insensitive substring match on key or value, newest first."""
        if not query:
            return ()
        q = query.lower()
        return tuple(e for e in self.list() if q in e.key.lower() or q in e.value.lower())[:limit]


class InMemoryMemoryStore(MemoryStore):
    def __init__(self) -> None:
        self._d: dict[str, MemoryEntry] = {}

    def store(self, key: str, value: str) -> MemoryEntry:
        _check_key(key)
        self._d[key] = MemoryEntry(key, value, time.time())
        return self._d[key]

    def view(self, key: str) -> MemoryEntry | None:
        _check_key(key)
        return self._d.get(key)

    def list(self) -> tuple[MemoryEntry, ...]:
        return tuple(sorted(self._d.values(), key=lambda e: e.created_at, reverse=True))

    def delete(self, key: str) -> bool:
        _check_key(key)
        return self._d.pop(key, None) is not None

    def clear(self) -> None:
        self._d.clear()


class FileMemoryStore(MemoryStore):
    def __init__(self, root: Path | str) -> None:
        self._root = Path(root)
        self._root.mkdir(parents=True, exist_ok=True)

    @property
    def root(self) -> Path:
        return self._root

    def _paths(self, key: str) -> tuple[Path, Path]:
        _check_key(key)
        return self._root / f"{key}.md", self._root / f"{key}.meta"

    def store(self, key: str, value: str) -> MemoryEntry:
        body, meta = self._paths(key)
        ts = time.time()
        body.write_text(value, encoding="utf-8")
        meta.write_text(json.dumps({"created_at": ts}), encoding="utf-8")
        return MemoryEntry(key, value, ts)

    def view(self, key: str) -> MemoryEntry | None:
        body, meta = self._paths(key)
        if not body.is_file():
            return None
        try:
            ts = float(json.loads(meta.read_text(encoding="utf-8"))["created_at"])
        except (OSError, ValueError, KeyError):
            ts = 0.0
        return MemoryEntry(key, body.read_text(encoding="utf-8"), ts)

    def list(self) -> tuple[MemoryEntry, ...]:
        es = [e for p in self._root.glob("*.md") if KEY_PATTERN.match(p.stem) and (e := self.view(p.stem))]
        return tuple(sorted(es, key=lambda e: e.created_at, reverse=True))

    def delete(self, key: str) -> bool:
        body, meta = self._paths(key)
        existed = body.is_file()
        body.unlink(missing_ok=True)
        meta.unlink(missing_ok=True)
        return existed

    def clear(self) -> None:
        for p in self._root.iterdir():
            if p.is_file() and p.suffix in (".md", ".meta"):
                p.unlink(missing_ok=True)


def memory_tools(store: MemoryStore, *, name_prefix: str = "memory_") -> tuple[Tool, ...]:
    obj = {"type": "object"}
    key_only = {**obj, "properties": {"key": {"type": "string"}}, "required": ["key"]}

    def view(*, key: str, **_: Any) -> str:
        e = store.view(key)
        return e.value if e is not None else "no entry"

    def put(*, key: str, value: str, **_: Any) -> str:
        store.store(key, value)
        return "ok"

    def recall(*, query: str, limit: int = 5, **_: Any) -> str:
        return "\n".join(f"{e.key}: {e.value.replace(chr(10), ' ').strip()}"
                         for e in store.recall(query, limit=int(limit)))

    def delete(*, key: str, **_: Any) -> str:
        return "deleted" if store.delete(key) else "no entry"

    return (
        FunctionTool(ToolSpec(f"{name_prefix}view", "Read a memory entry by key. Returns the stored value, or the "
                              "literal text 'no entry' if the key is unknown.", key_only), view),
        FunctionTool(ToolSpec(f"{name_prefix}store", "Insert or overwrite a memory entry. Keys must be alphanumeric "
                              "(with '.', '-', '_'). Returns 'ok'.",
                              {**obj, "properties": {"key": {"type": "string"}, "value": {"type": "string"}},
                               "required": ["key", "value"]}), put),
        FunctionTool(ToolSpec(f"{name_prefix}recall", "Search memory entries by substring. Returns up to 'limit' "
                              "matches as 'key: value' lines, newest first; empty string if no match.",
                              {**obj, "properties": {"query": {"type": "string"},
                                                     "limit": {"type": "integer", "default": 5}},
                               "required": ["query"]}), recall),
        FunctionTool(ToolSpec(f"{name_prefix}delete", "Remove a memory entry by key. Returns 'deleted' if the key "
                              "existed, 'no entry' otherwise.", key_only), delete),
    )


def register_memory_tools(registry: ToolRegistry, store: MemoryStore, *, name_prefix: str = "memory_") -> None:
    for t in memory_tools(store, name_prefix=name_prefix):
        registry.register(t)


__all__ = ["FileMemoryStore", "InMemoryMemoryStore", "KEY_PATTERN", "MemoryEntry", "MemoryStore", "memory_tools",
           "register_memory_tools"]

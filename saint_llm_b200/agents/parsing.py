"""Tool calls in model output: ``<tool_call name=".." [id=".."]>{json args}</tool_call>`` tags
and fenced JSON blocks (one object or a list of ``{"name", "arguments"[, "id"]}``).  These
are the output formats the model is trained to emit (reference:
``saint_llm_agents/tool_call_parser.py``); ``auto`` returns tag hits then new fenced hits."""

from __future__ import annotations

import json
import re
import uuid
from collections.abc import Iterator
from typing import Any, Literal

from saint_llm_b200.agents.core import ToolCall

_TAG = re.compile(r"<tool_call\s+([^>]+)>(.*?)</tool_call>", re.DOTALL)
_ATTR = re.compile(r'(\w+)="([^"]*)"')
_FENCE = re.compile(r"```(?:json)?\s*\n(.+?)\n```", re.DOTALL)


def _new_id() -> str:
    return f"call_{uuid.uuid4().hex[:8]}"


def _bad(strict: bool, msg: str) -> None:
    if strict:
        raise ValueError(msg)


def _from_tags(text: str, strict: bool) -> Iterator[ToolCall]:
    for m in _TAG.finditer(text):
        attrs = dict(_ATTR.findall(m.group(1)))
        body = m.group(2).strip()
        name = attrs.get("name")
        if not name:
            _bad(strict, f"tool_call tag missing name: {m.group(0)!r}")
            continue
        try:
            args = json.loads(body) if body else {}
        except json.JSONDecodeError:
            _bad(strict, f"tool_call {name!r} has invalid JSON body: {body!r}")
            continue
        if not isinstance(args, dict):
            _bad(strict, f"tool_call {name!r} arguments must be a JSON object")
            continue
        yield ToolCall(id=attrs.get("id") or _new_id(), name=name, arguments=args)


def _from_fences(text: str, strict: bool) -> Iterator[ToolCall]:
    for m in _FENCE.finditer(text):
        try:
            payload = json.loads(m.group(1).strip())
        except json.JSONDecodeError:
            _bad(strict, f"json-fenced block has invalid JSON: {m.group(1)!r}")
            continue
        for item in payload if isinstance(payload, list) else [payload]:
            name = item.get("name") if isinstance(item, dict) else None
            args: Any = item.get("arguments", {}) if isinstance(item, dict) else None
            if not isinstance(item, dict) or not isinstance(name, str) or not name or not isinstance(args, dict):
                _bad(strict, f"malformed json-fenced tool call: {item!r}")
                continue
            yield ToolCall(id=str(item.get("id") or _new_id()), name=name, arguments=args)


def _key(c: ToolCall) -> tuple[str, str]:
    try:
        return c.name, json.dumps(c.arguments, sort_keys=True, default=str)
    except TypeError:
        return c.name, str(c.arguments)


def parse_tool_calls(text: str, *, fmt: Literal["xml", "json", "auto"] = "auto", strict: bool = False
                     ) -> list[ToolCall]:
    if fmt == "xml":
        return list(_from_tags(text, strict))
    if fmt == "json":
        return list(_from_fences(text, strict))
    if fmt != "auto":
        raise ValueError(f"unknown parser format {fmt!r}")
    out = list(_from_tags(text, strict))
    seen = {_key(c) for c in out}
    for c in _from_fences(text, strict):
        if _key(c) not in seen:
            seen.add(_key(c))
            out.append(c)
    return out


def format_tool_call(call: ToolCall) -> str:
    """Render a call in the tag format the parser reads."""
    return f'<tool_call name="{call.name}" id="{call.id}">{json.dumps(dict(call.arguments))}</tool_call>'


__all__ = ["format_tool_call", "parse_tool_calls"]

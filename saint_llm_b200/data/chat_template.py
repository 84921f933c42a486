"""Chat rendering: turns -> token ids + SFT loss mask.

The marker strings, the segment order (role prefix, effort marker, thinking block,
visible answer + suffix) and which segments are loss-active are the reference's chat
format (``saint_llm_data/chat_template.py:40-235``); a model trained on one renders the
same way here.  Note that ``mask_thinking=True`` means the thinking block IS trained on.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

from saint_llm_b200.data.tokenizer import Tokenizer

Role = Literal["system", "user", "assistant"]


@dataclass(frozen=True)
class ChatTemplate:
    system_prefix: str = "<|system|>\n"
    system_suffix: str = "\n<|/system|>\n"
    user_prefix: str = "<|user|>\n"
    user_suffix: str = "\n<|/user|>\n"
    assistant_prefix: str = "<|assistant|>\n"
    assistant_suffix: str = "\n<|/assistant|>\n"
    think_start_marker: str = "<|think_start|>"
    think_end_marker: str = "<|think_end|>"
    effort_prefix_template: str = "<|effort:{tier}|>"
    bos_text: str = ""

    def effort(self, tier: int) -> str:
        return self.effort_prefix_template.format(tier=tier)


@dataclass(frozen=True)
class ChatTurn:
    role: Role
    content: str
    thinking: str = ""
    effort_tier: int | None = None


@dataclass(frozen=True)
class RenderedChat:
    token_ids: list[int]
    loss_mask: list[int]
    text: str


class ChatBuilder:
    """Accumulates (text, loss-active) segments; shared by the text and multimodal renderers."""

    def __init__(self, tokenizer: Tokenizer) -> None:
        self.tok = tokenizer
        self.ids: list[int] = []
        self.mask: list[int] = []
        self.text: list[str] = []

    def add(self, text: str, active: bool) -> None:
        if not text:
            return
        ids = self.tok.encode(text)
        self.ids += ids
        self.mask += [int(active)] * len(ids)
        self.text.append(text)

    def add_ids(self, ids: list[int], text: str, active: bool = False) -> None:
        self.ids += ids
        self.mask += [int(active)] * len(ids)
        self.text.append(text)

    def system(self, tmpl: ChatTemplate, content: str) -> None:
        self.add(tmpl.system_prefix + content + tmpl.system_suffix, False)

    def assistant(self, tmpl: ChatTemplate, turn: ChatTurn | object, mask_thinking: bool) -> None:
        self.add(tmpl.assistant_prefix, False)
        tier = getattr(turn, "effort_tier", None)
        if tier is not None:
            self.add(tmpl.effort(tier), False)
        thinking = getattr(turn, "thinking", "")
        if thinking:
            self.add(tmpl.think_start_marker + thinking + tmpl.think_end_marker, mask_thinking)
        self.add(getattr(turn, "content") + tmpl.assistant_suffix, True)

    def finish(self, tmpl: ChatTemplate, turns: Sequence[object], add_generation_prompt: bool,
               append_eos: bool) -> None:
        if add_generation_prompt:
            tier = None
            for t in turns:
                if getattr(t, "role") == "assistant":
                    tier = getattr(t, "effort_tier", None)
            self.add(tmpl.assistant_prefix + (tmpl.effort(tier) if tier is not None else ""), False)
        if append_eos:
            last = getattr(turns[-1], "role") if turns else None
            self.add_ids([self.tok.eos_token_id], "<eos>", active=last == "assistant")


def render_chat(turns: Sequence[ChatTurn], tokenizer: Tokenizer, *, template: ChatTemplate | None = None,
                add_generation_prompt: bool = False, append_eos: bool = False,
                mask_thinking: bool = True) -> RenderedChat:
    tmpl = template or ChatTemplate()
    b = ChatBuilder(tokenizer)
    b.add(tmpl.bos_text, False)
    for turn in turns:
        if turn.role == "system":
            b.system(tmpl, turn.content)
        elif turn.role == "user":
            b.add(tmpl.user_prefix + turn.content + tmpl.user_suffix, False)
        elif turn.role == "assistant":
            b.assistant(tmpl, turn, mask_thinking)
        else:
            raise ValueError(f"unknown role: {turn.role!r}")
    b.finish(tmpl, turns, add_generation_prompt, append_eos)
    return RenderedChat(b.ids, b.mask, "".join(b.text))


__all__ = ["ChatBuilder", "ChatTemplate", "ChatTurn", "RenderedChat", "Role", "render_chat"]

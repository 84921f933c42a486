"""A policy backed by this framework's model: the history is rendered with the chat
template (tool results as user turns marked ``[tool <id>]``, the tool catalogue and the
call format in the system turn), the answer is decoded through the KV cache and tool calls
are parsed from it."""

from __future__ import annotations

import json
from collections.abc import Sequence

import torch
from torch import nn

from saint_llm_b200.agents.core import Message, ToolSpec
from saint_llm_b200.agents.parsing import parse_tool_calls
from saint_llm_b200.data.chat_template import ChatTemplate, ChatTurn, render_chat
from saint_llm_b200.data.tokenizer import Tokenizer
from saint_llm_b200.infer.generate import decode
from saint_llm_b200.infer.sampling import SamplingParams

TOOL_FORMAT_HINT = ('To call a tool, write <tool_call name="TOOL_NAME">{"arg": value}</tool_call>. '
                    "Available tools:")


def tools_prompt(tools: Sequence[ToolSpec]) -> str:
    if not tools:
        return ""
    return "\n".join([TOOL_FORMAT_HINT] + [f"- {t.name}: {t.description} parameters={json.dumps(dict(t.parameters))}"
                                           for t in tools])


def to_chat_turns(messages: Sequence[Message], tools: Sequence[ToolSpec]) -> list[ChatTurn]:
    turns: list[ChatTurn] = []
    sys_text = "\n\n".join(m.content for m in messages if m.role == "system")
    catalogue = tools_prompt(tools)
    if sys_text or catalogue:
        turns.append(ChatTurn("system", "\n\n".join(x for x in (sys_text, catalogue) if x)))
    for m in messages:
        if m.role == "assistant":
            turns.append(ChatTurn("assistant", m.content))
        elif m.role == "tool":
            turns.append(ChatTurn("user", f"[tool {m.tool_call_id}] {m.content}"))
        elif m.role != "system":
            turns.append(ChatTurn("user", m.content))
    return turns


class ModelPolicy:
    def __init__(self, model: nn.Module, tokenizer: Tokenizer, *, template: ChatTemplate | None = None,
                 max_new_tokens: int = 256, temperature: float = 0.0, top_p: float = 1.0,
                 seed: int | None = None) -> None:
        self.model, self.tokenizer = model, tokenizer
        self.template = template or ChatTemplate()
        self.max_new_tokens = max_new_tokens
        self.params = SamplingParams(temperature=temperature, top_p=top_p)
        self.seed = seed

    @torch.no_grad()
    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message:
        ids = render_chat(to_chat_turns(messages, tools), self.tokenizer, template=self.template,
                          add_generation_prompt=True).token_ids
        dev = next(self.model.parameters()).device
        prompt = torch.tensor([ids], device=dev)
        gen = torch.Generator(device=dev).manual_seed(self.seed) if self.seed is not None else None
        was = self.model.training
        self.model.eval()
        try:
            out = decode(self.model, prompt, max_new_tokens=self.max_new_tokens, params=self.params,
                         eos_token=self.tokenizer.eos_token_id, generator=gen, use_cache=True)
        finally:
            self.model.train(was)
        new = [t for t in out[0, len(ids):].tolist()]
        eos = self.tokenizer.eos_token_id
        if eos in new:
            new = new[:new.index(eos)]
        text = self.tokenizer.decode(new)
        suffix = self.template.assistant_suffix.strip()
        if suffix and suffix in text:
            text = text[:text.index(suffix)]
        text = text.strip()
        return Message(role="assistant", content=text, tool_calls=tuple(parse_tool_calls(text)))


__all__ = ["ModelPolicy", "TOOL_FORMAT_HINT", "to_chat_turns", "tools_prompt"]

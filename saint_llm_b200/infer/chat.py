"""Stateful chat sessions over the streaming decoders (reference:
``saint_llm_inference/chat_session.py:49-235``, ``multimodal_chat_session.py:48-235``).

The history is rendered with the chat template plus a generation prompt; each streamed
id is decoded to text; the finished answer (EOS excluded, stripped) is appended to the
history as an assistant turn.  ``effort_tier`` makes the generation prompt
``<assistant prefix><|effort:N|>``.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.data.chat_template import ChatTemplate, ChatTurn, render_chat
from saint_llm_b200.data.multimodal import TokenSlots
from saint_llm_b200.data.multimodal_chat import MultimodalChatTurn, render_multimodal_chat
from saint_llm_b200.data.tokenizer import Tokenizer
from saint_llm_b200.infer.streaming import stream_greedy_decode, stream_top_p_sample


@dataclass(frozen=True)
class GenerationConfig:
    max_new_tokens: int = 256
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int | None = None
    seed: int | None = None


class _SessionBase:
    def __init__(self, *, model: nn.Module, tokenizer: Tokenizer, template: ChatTemplate | None,
                 eos_token: int | None) -> None:
        self._model = model
        self._tokenizer = tokenizer
        self._template = template or ChatTemplate()
        self._eos = eos_token if eos_token is not None else tokenizer.eos_token_id
        self.history: list = []

    @property
    def _device(self) -> torch.device:
        return next(self._model.parameters()).device

    def _stream_ids(self, prompt: Tensor, cfg: GenerationConfig, **features: Tensor | None) -> Iterator[Tensor]:
        if cfg.temperature < 1.0e-8:
            return stream_greedy_decode(self._model, prompt, max_new_tokens=cfg.max_new_tokens, eos_token=self._eos,
                                        **features)
        gen = torch.Generator(device=prompt.device).manual_seed(cfg.seed) if cfg.seed is not None else None
        return stream_top_p_sample(self._model, prompt, max_new_tokens=cfg.max_new_tokens, p=cfg.top_p,
                                   temperature=cfg.temperature, top_k=cfg.top_k, eos_token=self._eos, generator=gen,
                                   **features)

    def _respond_stream(self, prompt_ids: list[int], cfg: GenerationConfig | None, make_turn,
                        **features: Tensor | None) -> Iterator[str]:
        cfg = cfg or GenerationConfig()
        prompt = torch.tensor([prompt_ids], dtype=torch.long, device=self._device)
        was_training = self._model.training
        self._model.eval()
        got: list[int] = []
        try:
            for tok in self._stream_ids(prompt, cfg, **features):
                t = int(tok.reshape(-1)[0])
                if t == self._eos:
                    break
                got.append(t)
                yield self._tokenizer.decode([t])
        finally:
            self._model.train(was_training)
        self.history.append(make_turn(self._tokenizer.decode(got).strip()))

    def _generation_prompt(self, effort_tier: int) -> str:
        """Assistant prefix followed by the requested effort marker."""
        return self._template.assistant_prefix + self._template.effort(effort_tier)

    def reset(self) -> None:
        self.history = []


class ChatSession(_SessionBase):
    def __init__(self, *, model: nn.Module, tokenizer: Tokenizer, template: ChatTemplate | None = None,
                 system: str = "", eos_token: int | None = None) -> None:
        super().__init__(model=model, tokenizer=tokenizer, template=template, eos_token=eos_token)
        if system:
            self.history.append(ChatTurn(role="system", content=system))

    def add_user(self, text: str) -> None:
        if not text:
            raise ValueError("user message must be non-empty")
        self.history.append(ChatTurn(role="user", content=text))

    def add_system(self, text: str) -> None:
        if not text:
            raise ValueError("system message must be non-empty")
        self.history.append(ChatTurn(role="system", content=text))

    def prompt_ids(self, effort_tier: int | None = None) -> list[int]:
        if not self.history:
            raise ValueError("history is empty; add_user() before responding")
        if effort_tier is None:
            return render_chat(self.history, self._tokenizer, template=self._template,
                               add_generation_prompt=True).token_ids
        ids = render_chat(self.history, self._tokenizer, template=self._template).token_ids
        return ids + self._tokenizer.encode(self._generation_prompt(effort_tier))

    def stream_response(self, *, cfg: GenerationConfig | None = None, effort_tier: int | None = None) -> Iterator[str]:
        ids = self.prompt_ids(effort_tier)
        yield from self._respond_stream(ids, cfg, lambda text: ChatTurn(role="assistant", content=text))

    def respond(self, *, cfg: GenerationConfig | None = None, effort_tier: int | None = None) -> str:
        return "".join(self.stream_response(cfg=cfg, effort_tier=effort_tier))


class MultimodalChatSession(_SessionBase):
    def __init__(self, *, model: nn.Module, tokenizer: Tokenizer, slots: TokenSlots,
                 template: ChatTemplate | None = None, system: str = "", eos_token: int | None = None) -> None:
        super().__init__(model=model, tokenizer=tokenizer, template=template, eos_token=eos_token)
        self._slots = slots
        if system:
            self.history.append(MultimodalChatTurn(role="system", content=system))

    def add_user(self, text: str = "", *, image_features: Sequence[Tensor] = (),
                 audio_features: Sequence[Tensor] = ()) -> None:
        if not text and not image_features and not audio_features:
            raise ValueError("user turn needs text or an attachment")
        self.history.append(MultimodalChatTurn(role="user", content=text, image_features=tuple(image_features),
                                               audio_features=tuple(audio_features)))

    def add_system(self, text: str) -> None:
        if not text:
            raise ValueError("system message must be non-empty")
        self.history.append(MultimodalChatTurn(role="system", content=text))

    def stream_response(self, *, cfg: GenerationConfig | None = None, effort_tier: int | None = None) -> Iterator[str]:
        if not self.history:
            raise ValueError("history is empty; add_user() before responding")
        r = render_multimodal_chat(self.history, self._tokenizer, self._slots, template=self._template,
                                   add_generation_prompt=effort_tier is None)
        ids = r.token_ids + (self._tokenizer.encode(self._generation_prompt(effort_tier)) if effort_tier is not None
                             else [])
        dev = self._device
        feats = {"vision_features": None if r.vision_features is None else r.vision_features.to(dev),
                 "audio_features": None if r.audio_features is None else r.audio_features.to(dev)}
        yield from self._respond_stream(ids, cfg, lambda text: MultimodalChatTurn(role="assistant", content=text),
                                        **feats)

    def respond(self, *, cfg: GenerationConfig | None = None, effort_tier: int | None = None) -> str:
        return "".join(self.stream_response(cfg=cfg, effort_tier=effort_tier))


__all__ = ["ChatSession", "GenerationConfig", "MultimodalChatSession"]

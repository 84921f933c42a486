"""Chat rendering with image/audio attachments (reference:
``saint_llm_data/multimodal_chat.py:41-287``): placeholders are woven inside the user turn's
role markers, features are stacked in render order (one row per model-filled slot)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch
from torch import Tensor

from saint_llm_b200.data.chat_template import ChatBuilder, ChatTemplate, ChatTurn, RenderedChat
from saint_llm_b200.data.multimodal import TokenSlots, audio_slot_rows
from saint_llm_b200.data.tokenizer import Tokenizer


@dataclass(frozen=True)
class MultimodalChatTurn:
    role: str
    content: str
    thinking: str = ""
    effort_tier: int | None = None
    image_features: tuple[Tensor, ...] = ()
    audio_features: tuple[Tensor, ...] = ()


@dataclass(frozen=True)
class RenderedMultimodalChat:
    token_ids: list[int]
    loss_mask: list[int]
    vision_features: Tensor | None = None
    audio_features: Tensor | None = None
    text: str = ""

    def to_torch(self, *, device: torch.device | None = None) -> tuple[Tensor, Tensor]:
        return (torch.tensor([self.token_ids], dtype=torch.long, device=device),
                torch.tensor([self.loss_mask], dtype=torch.long, device=device))


def render_multimodal_chat(turns: Sequence[MultimodalChatTurn], tokenizer: Tokenizer, slots: TokenSlots, *,
                           template: ChatTemplate | None = None, add_generation_prompt: bool = False,
                           append_eos: bool = False, mask_thinking: bool = True) -> RenderedMultimodalChat:
    tmpl = template or ChatTemplate()
    b = ChatBuilder(tokenizer)
    vis: list[Tensor] = []
    aud: list[Tensor] = []
    b.add(tmpl.bos_text, False)
    for t in turns:
        if t.role == "system":
            b.system(tmpl, t.content)
        elif t.role == "user":
            b.add(tmpl.user_prefix, False)
            b.add(t.content, False)
            for img in t.image_features:
                if img.dim() != 2:
                    raise ValueError(f"image features must be (n_patches, dim); got {tuple(img.shape)}")
                b.add_ids([slots.image_pad] * img.shape[0], "<image_pad>" * img.shape[0])
                vis.append(img)
            for clip in t.audio_features:
                if clip.dim() != 2:
                    raise ValueError(f"audio features must be (n_tokens, dim); got {tuple(clip.shape)}")
                b.add_ids([slots.audio_start] * (clip.shape[0] + 1) + [slots.audio_end], f"<audio:{clip.shape[0]}>")
                aud.append(audio_slot_rows(clip))
            b.add(tmpl.user_suffix, False)
        elif t.role == "assistant":
            b.assistant(tmpl, t, mask_thinking)
        else:
            raise ValueError(f"unknown role: {t.role!r}")
    b.finish(tmpl, turns, add_generation_prompt, append_eos)
    return RenderedMultimodalChat(b.ids, b.mask, torch.cat(vis) if vis else None, torch.cat(aud) if aud else None,
                                  "".join(b.text))


def to_chat_turn(turn: MultimodalChatTurn) -> ChatTurn:
    return ChatTurn(role=turn.role, content=turn.content, thinking=turn.thinking,  # type: ignore[arg-type]
                    effort_tier=turn.effort_tier)


def render_text_chat_to_multimodal(chat: RenderedChat) -> RenderedMultimodalChat:
    return RenderedMultimodalChat(chat.token_ids, chat.loss_mask, None, None, chat.text)


__all__ = ["MultimodalChatTurn", "RenderedMultimodalChat", "render_multimodal_chat", "render_text_chat_to_multimodal",
           "to_chat_turn"]

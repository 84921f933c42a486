"""Chat rendering and multimodal encoding on CPU: which segments carry loss, where the
placeholder slots sit, and how feature rows line up with them."""

from __future__ import annotations

import pytest
import torch

from saint_llm_b200.data.chat_template import ChatTemplate, ChatTurn, render_chat
from saint_llm_b200.data.multimodal import (MultimodalExample, TokenSlots, audio_slot_rows,
                                            encode_multimodal)
from saint_llm_b200.data.multimodal_chat import (MultimodalChatTurn, render_multimodal_chat,
                                                 render_text_chat_to_multimodal, to_chat_turn)
from saint_llm_b200.data.tokenizer import CharTokenizer

TOK = CharTokenizer()
SLOTS = TokenSlots(image_pad=3, audio_start=4, audio_end=5)


def _active_text(ids, mask):
    return TOK.decode([i for i, m in zip(ids, mask) if m])


def test_render_chat_loss_segments():
    t = ChatTemplate()
    turns = [ChatTurn("system", "be brief"), ChatTurn("user", "2+2?"),
             ChatTurn("assistant", "4", thinking="add", effort_tier=2)]
    r = render_chat(turns, TOK, append_eos=True)
    assert len(r.token_ids) == len(r.loss_mask)
    # thinking (mask_thinking=True trains on it), the answer with its suffix, and the EOS
    assert _active_text(r.token_ids, r.loss_mask) == (t.think_start_marker + "add" + t.think_end_marker
                                                      + "4" + t.assistant_suffix)
    assert r.token_ids[-1] == TOK.eos_token_id and r.loss_mask[-1] == 1
    assert TOK.decode(r.token_ids) + "<eos>" == r.text
    assert t.effort(2) in r.text and "<|effort:2|>" in r.text
    no_think = render_chat(turns, TOK, mask_thinking=False)
    assert _active_text(no_think.token_ids, no_think.loss_mask) == "4" + t.assistant_suffix


def test_render_chat_generation_prompt_and_eos_rules():
    t = ChatTemplate()
    turns = [ChatTurn("assistant", "a", effort_tier=1), ChatTurn("user", "q")]
    r = render_chat(turns, TOK, add_generation_prompt=True, append_eos=True)
    # the generation prompt repeats the last assistant effort tier; EOS after a user turn is not trained
    assert r.text.endswith(t.assistant_prefix + t.effort(1) + "<eos>")
    assert r.loss_mask[-1] == 0
    assert render_chat([], TOK).token_ids == []
    with pytest.raises(ValueError):
        render_chat([ChatTurn("tool", "x")], TOK)  # type: ignore[arg-type]
    custom = render_chat([ChatTurn("user", "hi")], TOK, template=ChatTemplate(user_prefix="U:", user_suffix="|",
                                                                             bos_text="^"))
    assert custom.text == "^U:hi|" and sum(custom.loss_mask) == 0


def test_text_only_multimodal_chat_equals_the_text_renderer():
    mm = [MultimodalChatTurn("system", "s"), MultimodalChatTurn("user", "u"),
          MultimodalChatTurn("assistant", "a", thinking="t", effort_tier=0)]
    a = render_multimodal_chat(mm, TOK, SLOTS, append_eos=True, add_generation_prompt=False)
    b = render_chat([to_chat_turn(x) for x in mm], TOK, append_eos=True)
    assert a.token_ids == b.token_ids and a.loss_mask == b.loss_mask
    assert a.vision_features is None and a.audio_features is None
    c = render_text_chat_to_multimodal(b)
    assert c.token_ids == b.token_ids and c.text == b.text
    ids, mask = a.to_torch()
    assert ids.shape == mask.shape == (1, len(b.token_ids)) and ids.dtype == torch.long


def test_multimodal_chat_slots_sit_inside_the_user_turn():
    t = ChatTemplate()
    img = torch.randn(2, 6)
    clip = torch.randn(3, 6)
    r = render_multimodal_chat([MultimodalChatTurn("user", "see", image_features=(img,), audio_features=(clip,)),
                                MultimodalChatTurn("assistant", "ok")], TOK, SLOTS)
    ids = r.token_ids
    pre = len(TOK.encode(t.user_prefix + "see"))
    assert ids[pre:pre + 2] == [3, 3]                    # one pad per patch
    assert ids[pre + 2:pre + 7] == [4, 4, 4, 4, 5]       # start x (n + 1), end
    assert TOK.decode(ids[pre + 7:pre + 7 + len(t.user_suffix)]) == t.user_suffix
    assert torch.equal(r.vision_features, img)
    assert r.audio_features.shape == (5, 6) and torch.equal(r.audio_features[1:4], clip)
    assert not r.audio_features[0].any() and not r.audio_features[4].any()
    assert sum(r.loss_mask[:pre + 7]) == 0
    for bad in (dict(image_features=(torch.randn(6),)), dict(audio_features=(torch.randn(1, 2, 3),))):
        with pytest.raises(ValueError):
            render_multimodal_chat([MultimodalChatTurn("user", "x", **bad)], TOK, SLOTS)


def test_encode_multimodal_layout_and_mask():
    ex = MultimodalExample("p", "r", image_features=(torch.zeros(2, 4), torch.zeros(1, 4)),
                           audio_features=(torch.zeros(2, 4),))
    ids, mask = encode_multimodal(ex, TOK, SLOTS)
    p = TOK.encode("p")
    assert ids == p + [3, 3, 3] + [4, 4, 4, 5] + TOK.encode("r") + [TOK.eos_token_id]
    assert mask == [0] * (len(p) + 7) + [1, 1]
    ids2, mask2 = encode_multimodal(ex, TOK, SLOTS, append_eos=False)
    assert ids2 == ids[:-1] and mask2 == mask[:-1]
    rows = audio_slot_rows(torch.ones(2, 3))
    assert rows.shape == (4, 3) and rows[0].sum() == 0 and rows[-1].sum() == 0 and rows[1:3].eq(1).all()


def test_token_slots_lookup_errors():
    with pytest.raises(ValueError, match="missing special tokens"):
        TokenSlots.from_tokenizer(TOK)  # a character tokenizer has no named specials
    with pytest.raises(ValueError, match="cannot look up"):
        TokenSlots.from_tokenizer(object())  # type: ignore[arg-type]

    class _Named:
        def token_to_id(self, t):
            return {"<|image_pad|>": 7, "<|audio_start|>": 8, "<|audio_end|>": 9}.get(t)

    assert TokenSlots.from_tokenizer(_Named()) == TokenSlots(7, 8, 9)  # type: ignore[arg-type]

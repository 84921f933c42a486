"""Supervised fine-tuning on CPU: the JSONL dataset, the response-masked loss straight from the
model against the logits path, and the multimodal SFT step with spliced features."""

import json

import pytest
import torch

from saint_llm_b200.config import ModelConfig, MultimodalConfig
from saint_llm_b200.data.multimodal import MultimodalExample, TokenSlots, pack_multimodal_examples
from saint_llm_b200.data.tokenizer import CharTokenizer
from saint_llm_b200.models import SaintLLM
from saint_llm_b200.posttrain.sft import (JsonlSFTDataset, SFTExample, encode_sft, masked_next_token_ce,
                                          multimodal_sft_step, sft_loss)

TOK = CharTokenizer(base_vocab=16, unicode_max=480)


def test_jsonl_dataset_skips_bad_rows_and_keeps_system(tmp_path):
    path = tmp_path / "sft.jsonl"
    rows = [{"prompt": "ab", "response": "cd", "system": "s"}, "not json", {"prompt": "x"},
            {"prompt": 3, "response": "y"}, {"q": "ef", "a": "gh"}, {"prompt": "ij", "response": "kl"}]
    path.write_text("\n".join(r if isinstance(r, str) else json.dumps(r) for r in rows) + "\n\n")
    ds = JsonlSFTDataset(path, tokenizer=TOK, seq_len=4, batch_size=1, drop_last=False)
    toks = torch.cat([b.tokens.reshape(-1) for b in ds])
    want = encode_sft(SFTExample("ab", "cd", "s"), TOK)[0] + encode_sft(SFTExample("ij", "kl"), TOK)[0]
    assert toks[:len(want)].tolist() == want
    custom = JsonlSFTDataset(path, tokenizer=TOK, seq_len=4, prompt_field="q", response_field="a",
                             system_field=None, drop_last=False)
    got = torch.cat([b.tokens.reshape(-1) for b in custom])
    w2 = encode_sft(SFTExample("ef", "gh"), TOK)[0]
    assert got[:len(w2)].tolist() == w2
    with pytest.raises(FileNotFoundError):
        JsonlSFTDataset(tmp_path / "missing.jsonl", tokenizer=TOK, seq_len=4)


def test_sft_loss_from_the_model_equals_masked_ce_of_its_logits():
    torch.manual_seed(0)
    m = SaintLLM(ModelConfig.tiny()).eval()
    g = torch.Generator().manual_seed(1)
    tokens = torch.randint(0, 480, (2, 12), generator=g)
    mask = torch.zeros(2, 12, dtype=torch.long)
    mask[:, 7:] = 1
    mask[1, 10:] = 0
    with torch.no_grad():
        want, n = masked_next_token_ce(m(tokens)["logits"], tokens, mask)
        got = sft_loss(m, tokens, mask)
    assert n == 5 + 3
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    empty = torch.zeros_like(mask)
    with torch.no_grad():
        assert float(sft_loss(m, tokens, empty)) == 0.0  # no response token: zero, not NaN


def test_multimodal_sft_step_splices_the_window_features():
    cfg = ModelConfig.tiny().model_copy(update={"multimodal": MultimodalConfig(enable_vision_projector=True,
                                                                               vision_input_dim=8)})
    torch.manual_seed(0)
    m = SaintLLM(cfg)
    slots = TokenSlots.from_model_config(cfg)
    g = torch.Generator().manual_seed(3)
    exs = [MultimodalExample("look", "cat", image_features=(torch.randn(3, 8, generator=g),)),
           MultimodalExample("and", "dog", image_features=(torch.randn(2, 8, generator=g),))]
    wins = list(pack_multimodal_examples(exs, TOK, slots, seq_len=10, drop_last=False))
    for w in wins:
        out = multimodal_sft_step(m, w)
        n_img = int((w.tokens == slots.image_pad).sum())
        assert (w.vision_features is None) == (n_img == 0)
        assert out.n_response_tokens == int(w.loss_mask[:, 1:].sum())
        assert torch.isfinite(out.loss) and out.logits_for_aux is not None
    w = next(w for w in wins if w.vision_features is not None)
    out = multimodal_sft_step(m, w)
    out.loss.backward()
    assert m.vision_proj.up.weight.grad is not None and m.vision_proj.up.weight.grad.any()  # features reached the model

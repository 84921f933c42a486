"""Generative-reward judge arithmetic, reward scoring, frozen log-probs and the multimodal
row selection of GRPO on CPU, with stub language models."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch
from torch import nn

from saint_llm_b200.posttrain.grm import (GRMConfig, GRMRewardFn, binary_grm_config, judge_completion,
                                          likert_grm_config)
from saint_llm_b200.posttrain.grpo import GRPOConfig
from saint_llm_b200.posttrain.multimodal_grpo import (MultimodalRolloutBatch, multimodal_grpo_train_step,
                                                      select_rows)
from saint_llm_b200.posttrain.trainer import frozen_logprobs, score_rollouts


class _BigramLM(nn.Module):
    """logits[b, t] = table[tokens[b, t]]: a model whose outputs are easy to write down."""

    def __init__(self, vocab: int = 12, seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.table = nn.Parameter(torch.randn(vocab, vocab, generator=g))
        self.seen_training: list[bool] = []

    def forward(self, ids, **_):
        self.seen_training.append(self.training)
        return {"logits": self.table[ids]}


def test_judge_is_the_expected_score_under_renormalised_verdicts():
    lm = _BigramLM()
    ids = torch.tensor([[3, 4, 5], [1, 2, 9]])
    cfg = GRMConfig("{prompt}{completion}", (7, 2, 10), (1.0, 0.25, 0.0), temperature=0.5)
    got = judge_completion(lm, ids, cfg)
    last = lm.table[ids[:, -1]][:, [7, 2, 10]] / 0.5
    want = torch.softmax(last, -1) @ torch.tensor([1.0, 0.25, 0.0])
    torch.testing.assert_close(got, want)
    with pytest.raises(ValueError):
        judge_completion(lm, ids[0], cfg)


def test_grm_configs():
    b = binary_grm_config(good_token_id=4, bad_token_id=5)
    assert b.score_token_ids == (4, 5) and b.score_values == (1.0, 0.0)
    lk = likert_grm_config(score_token_ids=[1, 2, 3, 4, 5], prompt_template="{prompt}{completion}")
    assert lk.score_values == (0.0, 0.25, 0.5, 0.75, 1.0)
    with pytest.raises(ValueError):
        likert_grm_config(score_token_ids=[1], prompt_template="x")
    for bad in (dict(score_token_ids=(1, 2), score_values=(1.0,)), dict(score_token_ids=(), score_values=()),
                dict(score_token_ids=(1,), score_values=(1.0,), temperature=0.0)):
        with pytest.raises(ValueError):
            GRMConfig("t", **bad)


def test_grm_reward_fn_formats_encodes_and_restores_training_mode():
    lm = _BigramLM().train()
    seen = []

    def encode(text):
        seen.append(text)
        return [ord(c) % 12 for c in text]

    fn = GRMRewardFn(lm, encode, binary_grm_config(good_token_id=1, bad_token_id=2, prompt_template="P={prompt};C={completion}"))
    r = fn("ab", "cd")
    assert seen == ["P=ab;C=cd"] and 0.0 <= r <= 1.0
    assert lm.seen_training == [False] and lm.training  # judged in eval mode, mode restored
    with pytest.raises(ValueError):
        GRMRewardFn(lm, lambda s: [], binary_grm_config(good_token_id=1, bad_token_id=2))("a", "b")


def test_score_rollouts():
    r = score_rollouts(prompts=["a", "bb"], completions=["xyz", "q"], reward_fn=lambda p, c: len(p) + len(c))
    assert r.dtype == torch.float32 and r.tolist() == [4.0, 3.0]
    with pytest.raises(ValueError):
        score_rollouts(prompts=["a"], completions=[], reward_fn=lambda p, c: 0.0)


def test_frozen_logprobs_are_detached_and_keep_the_mode():
    lm = _BigramLM().train()
    ids = torch.tensor([[1, 2, 3, 4]])
    lp = frozen_logprobs(lm, ids)
    assert not lp.requires_grad and lm.training and lm.seen_training == [False]
    want = torch.log_softmax(lm.table[ids[:, :-1]], -1).gather(-1, ids[:, 1:, None]).squeeze(-1)
    torch.testing.assert_close(lp[:, 1:], want.detach())
    assert lp[0, 0] == 0


# ------------------------------------------------------------ multimodal selection
SLOTS = SimpleNamespace(image_pad=11, audio_start=8, audio_end=9)


def _mm_batch():
    # rows 0..3: row 0 has 2 image slots, row 1 none, row 2 one, row 3 two; audio slots in rows 1 and 3
    tokens = torch.tensor([[11, 11, 1, 2],
                           [8, 1, 9, 3],
                           [1, 11, 2, 3],
                           [11, 8, 11, 4]])
    n_img = int((tokens == 11).sum())
    n_aud = int(((tokens >= 8) & (tokens <= 9)).sum())
    vis = torch.arange(n_img, dtype=torch.float32)[:, None].expand(n_img, 3).clone()
    aud = 100 + torch.arange(n_aud, dtype=torch.float32)[:, None]
    z = torch.zeros(4, 4)
    return MultimodalRolloutBatch(tokens, torch.ones_like(tokens), z, z, torch.tensor([1.0, 0.0, 1.0, 1.0]), vis, aud)


def test_select_rows_keeps_the_feature_rows_of_the_kept_slots():
    b = _mm_batch()
    out = select_rows(b, torch.tensor([False, True, False, True]), SLOTS)
    assert out.tokens.tolist() == [[8, 1, 9, 3], [11, 8, 11, 4]]
    # image features in slot order: row0 -> 0, 1; row2 -> 2; row3 -> 3, 4
    assert out.vision_features[:, 0].tolist() == [3.0, 4.0]
    # audio features: row1 -> 100, 101; row3 -> 102
    assert out.audio_features[:, 0].tolist() == [100.0, 101.0, 102.0]
    assert out.rewards.tolist() == [0.0, 1.0]
    none = select_rows(MultimodalRolloutBatch(*[getattr(b, f) for f in ("tokens", "response_mask", "old_logprobs",
                                                                         "ref_logprobs", "rewards")]),
                       torch.tensor([True, False, True, False]), SLOTS)
    assert none.vision_features is None and none.audio_features is None


def test_multimodal_step_without_signal_returns_zero_loss():
    b = _mm_batch()
    flat = MultimodalRolloutBatch(b.tokens, b.response_mask, b.old_logprobs, b.ref_logprobs, torch.ones(4),
                                  b.vision_features, b.audio_features)
    lm = _BigramLM()
    opt = torch.optim.SGD(lm.parameters(), lr=1.0)
    before = lm.table.detach().clone()
    out = multimodal_grpo_train_step(actor=lm, optimizer=opt, batch=flat, cfg=GRPOConfig(group_size=2))
    assert out.n_kept_groups == 0 and float(out.loss.detach()) == 0.0 and float(out.metrics["reward_mean"]) == 1.0
    assert torch.equal(lm.table, before) and lm.seen_training == []

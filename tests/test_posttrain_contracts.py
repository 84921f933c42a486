"""Post-training helper contracts on CPU: SFT encoding, packing and masked losses, on-policy
distillation (teacher pooling, KL), ThinkPRM step boundaries / scores / filter, critique
masks."""

import math

import pytest
import torch

from saint_llm_b200.data.tokenizer import CharTokenizer
from saint_llm_b200.posttrain.critique import needs_critique_mask
from saint_llm_b200.posttrain.opd import aggregate_teacher_logits, opd_kl_loss
from saint_llm_b200.posttrain.sft import (
    SFTExample,
    encode_sft,
    masked_next_token_ce,
    pack_sft_examples,
    pack_sft_into_batch,
)
from saint_llm_b200.posttrain.think_prm import (
    StepRewardHead,
    find_step_boundaries,
    gather_step_scores,
    prm_filter_mask,
    step_prm_loss,
)


# --------------------------------------------------------------------- SFT
def test_encode_sft_masks_only_the_response():
    tok = CharTokenizer()
    ids, mask = encode_sft(SFTExample("hi", "yo", system="s"), tok)
    assert len(ids) == len(mask) == len("s\nhi") + len("yo") + 1
    assert mask == [0] * 4 + [1] * 3 and ids[-1] == tok.eos_token_id
    ids2, mask2 = encode_sft(SFTExample("hi", "yo"), tok, append_eos=False)
    assert mask2 == [0, 0, 1, 1] and tok.eos_token_id not in ids2[-1:]


def test_sft_packing_keeps_masks_aligned_and_pads():
    tok = CharTokenizer()
    exs = [SFTExample("abc", "de"), SFTExample("f", "ghij"), SFTExample("k", "l")]
    wins = list(pack_sft_examples(exs, tok, seq_len=5, drop_last=False, pad_token_id=0))
    toks = torch.cat([w.tokens[0] for w in wins])
    mask = torch.cat([w.loss_mask[0] for w in wins])
    seg = torch.cat([w.segment_ids[0] for w in wins])
    flat_ids, flat_mask = [], []
    for e in exs:
        i, m = encode_sft(e, tok)
        flat_ids += i
        flat_mask += m
    n = len(flat_ids)
    assert toks[:n].tolist() == flat_ids and mask[:n].tolist() == flat_mask
    assert (mask[n:] == 0).all() and seg[:n].tolist() == sorted(seg[:n].tolist())
    batches = list(pack_sft_into_batch(exs, tok, batch_size=2, seq_len=5, drop_last=False))
    last = batches[-1]
    assert last.tokens.shape == (2, 5)
    if (last.segment_ids == -1).any():
        assert (last.loss_mask[last.segment_ids == -1] == 0).all()
    with pytest.raises(ValueError):
        list(pack_sft_examples(exs, tok, seq_len=0))


def test_masked_next_token_ce_counts_only_masked_targets():
    torch.manual_seed(0)
    logits = torch.randn(2, 4, 6)
    toks = torch.randint(0, 6, (2, 4))
    mask = torch.tensor([[0, 0, 1, 1], [0, 1, 0, 0]])
    loss, n = masked_next_token_ce(logits, toks, mask)
    assert n == 3
    lp = torch.log_softmax(logits[:, :-1], -1).gather(-1, toks[:, 1:, None])[..., 0]
    want = -(lp[0, 1] + lp[0, 2] + lp[1, 0]) / 3
    torch.testing.assert_close(loss, want)
    zero, n0 = masked_next_token_ce(logits, toks, torch.zeros_like(mask))
    assert n0 == 0 and zero.item() == 0.0


# --------------------------------------------------------------------- OPD
def test_teacher_pooling_modes():
    torch.manual_seed(1)
    a, b = torch.randn(1, 2, 5), torch.randn(1, 2, 5)
    mean = aggregate_teacher_logits([a, b])
    want = torch.log(0.5 * torch.softmax(a, -1) + 0.5 * torch.softmax(b, -1))
    torch.testing.assert_close(mean, want, rtol=1e-5, atol=1e-5)
    w = aggregate_teacher_logits([a, b], weights=torch.tensor([1.0, 0.0]), mode="weighted")
    torch.testing.assert_close(w, torch.log_softmax(a, -1), rtol=1e-4, atol=1e-4)
    mx = aggregate_teacher_logits([a, a + 10.0 * (torch.arange(5) == 0)], mode="max")
    torch.testing.assert_close(mx.exp().sum(-1), torch.ones(1, 2))
    for kw in ({"mode": "weighted"}, {"mode": "weighted", "weights": torch.tensor([0.7, 0.7])},
               {"mode": "median"}):
        with pytest.raises(ValueError):
            aggregate_teacher_logits([a, b], **kw)
    with pytest.raises(ValueError):
        aggregate_teacher_logits([])


def test_opd_kl_is_zero_for_identical_and_positive_otherwise():
    torch.manual_seed(2)
    s = torch.randn(2, 3, 7)
    mask = torch.tensor([[1, 1, 0], [0, 1, 1]])
    kl0, n = opd_kl_loss(s, torch.log_softmax(s, -1), mask)
    assert n == 4 and abs(kl0.item()) < 1e-6
    kl1, _ = opd_kl_loss(s, torch.log_softmax(torch.randn(2, 3, 7), -1), mask, chunk_rows=2)
    assert kl1.item() > 0
    # chunking does not change the value
    kl2, _ = opd_kl_loss(s, torch.log_softmax(s * 0.5, -1), mask, chunk_rows=1)
    kl3, _ = opd_kl_loss(s, torch.log_softmax(s * 0.5, -1), mask, chunk_rows=100)
    torch.testing.assert_close(kl2, kl3)
    with pytest.raises(ValueError):
        opd_kl_loss(s, torch.log_softmax(s, -1), mask, temperature=0.0)


# ---------------------------------------------------------------- ThinkPRM
def test_step_boundaries_scores_and_filter():
    toks = torch.tensor([[5, 9, 5, 5, 9, 9], [1, 2, 3, 4, 5, 6]])
    pos = find_step_boundaries(toks, 9)
    assert pos[0, :3].tolist() == [1, 4, 5] and (pos[0, 3:] == -1).all() and (pos[1] == -1).all()
    torch.manual_seed(3)
    from saint_llm_b200.posttrain.think_prm import ThinkPRMConfig

    head = StepRewardHead(ThinkPRMConfig(hidden_dim=4))
    hidden = torch.randn(2, 6, 4)
    probs, valid = gather_step_scores(hidden, head, pos)
    assert valid.sum().item() == 3 and (probs[~valid] == 0).all() and ((probs[valid] > 0) & (probs[valid] < 1)).all()
    keep = prm_filter_mask(probs, valid, min_score=0.0)
    assert keep.all()  # nothing scores below 0; the step-less row is kept
    strict = prm_filter_mask(probs, valid, min_score=1.0)
    assert strict.tolist() == [False, True]
    logits = torch.tensor([[2.0, -1.0, 0.0]])
    labels = torch.tensor([[1, 0, 1]])
    mask = torch.tensor([[1, 1, 0]])
    want = (math.log1p(math.exp(-2.0)) + math.log1p(math.exp(-1.0))) / 2
    assert step_prm_loss(logits, labels, mask).item() == pytest.approx(want, rel=1e-5)
    with pytest.raises(ValueError):
        step_prm_loss(logits, labels[:, :2], mask)


def test_critique_mask_threshold():
    r = torch.tensor([0.1, 0.9, 0.5, -1.0])
    assert needs_critique_mask(r, threshold=0.5).tolist() == [True, False, False, True]

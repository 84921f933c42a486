"""Post-training math and drivers on CPU, against the unmodified reference where it exists."""

import dataclasses

import pytest
import torch

from saint_llm_b200.config import ModelConfig
from saint_llm_b200.data import CharTokenizer
from saint_llm_b200.models import SaintLLM
from saint_llm_b200.posttrain import (
    GRPOConfig,
    GTPOConfig,
    OPDConfig,
    RolloutBatch,
    RolloutGenConfig,
    SFTExample,
    SpecialistPipeline,
    StepRewardHead,
    ThinkPRMConfig,
    TreeRolloutBatch,
    aggregate_teacher_logits,
    binary_grm_config,
    build_rollout_batch,
    collect_critique_requests,
    compute_tree_advantage,
    decode_rollouts_for_reward,
    find_step_boundaries,
    generate_grpo_rollouts,
    grpo_loss,
    grpo_train_step,
    gtpo_loss,
    judge_completion,
    length_target_reward,
    opd_kl_loss,
    pack_sft_into_batch,
    policy_token_logprobs,
    sft_cross_entropy,
    sft_loss,
    tree_dynamic_sampling_mask,
    tree_grpo_loss,
    unigram_overlap_reward,
)


def _batch(seed=0, b=2, g=4, t=12, v=50):
    gen = torch.Generator().manual_seed(seed)
    n = b * g
    tokens = torch.randint(0, v, (n, t), generator=gen)
    mask = torch.zeros(n, t, dtype=torch.long)
    mask[:, 5:] = 1
    mask[0, 10:] = 0
    old = -torch.rand(n, t, generator=gen)
    ref = -torch.rand(n, t, generator=gen)
    rewards = torch.randint(0, 2, (n,), generator=gen).float()
    rewards[:g] = 1.0  # a zero-variance group
    logits = torch.randn(n, t, v, generator=gen, requires_grad=True)
    return logits, tokens, mask, old, ref, rewards


CFGS = [GRPOConfig(group_size=4), GRPOConfig(group_size=4, importance_ratio_level="sequence"),
        GRPOConfig(group_size=4, use_clip_higher=True, token_level_pg=True),
        GRPOConfig(group_size=4, unbiased_loss=True, kl_coef=0.1)]


@pytest.mark.parametrize("cfg", CFGS)
def test_grpo_loss_matches_reference(ref_pkgs, cfg):
    from saint_llm_posttraining import grpo as rg

    logits, tokens, mask, old, ref, rewards = _batch()
    ours, m1 = grpo_loss(logits, RolloutBatch(tokens, mask, old, ref, rewards), cfg=cfg)
    rcfg = rg.GRPOConfig(**dataclasses.asdict(cfg))
    theirs, m2 = rg.grpo_loss(logits, rg.RolloutBatch(tokens, mask, old, ref, rewards), cfg=rcfg)
    torch.testing.assert_close(ours, theirs, rtol=1e-5, atol=1e-6)
    g1 = torch.autograd.grad(ours, logits)[0]
    g2 = torch.autograd.grad(theirs, logits)[0]
    torch.testing.assert_close(g1, g2, rtol=1e-4, atol=1e-6)
    for k in m2:
        torch.testing.assert_close(m1[k].float(), m2[k].float(), rtol=1e-5, atol=1e-6)


def test_gtpo_and_tree_match_reference(ref_pkgs):
    from saint_llm_posttraining import grpo as rg
    from saint_llm_posttraining import gtpo as rgt
    from saint_llm_posttraining import tree_grpo as rtr

    logits, tokens, mask, old, ref, rewards = _batch(1)
    cfg = GTPOConfig(grpo=GRPOConfig(group_size=4), entropy_alpha=0.7)
    ours, _ = gtpo_loss(logits, RolloutBatch(tokens, mask, old, ref, rewards), cfg=cfg)
    theirs, _ = rgt.gtpo_loss(logits, rg.RolloutBatch(tokens, mask, old, ref, rewards),
                              cfg=rgt.GTPOConfig(grpo=rg.GRPOConfig(group_size=4), entropy_alpha=0.7))
    torch.testing.assert_close(ours, theirs, rtol=1e-5, atol=1e-6)
    parent = torch.tensor([-1, -1, 0, 0, 0, 1, 2, 2])
    torch.testing.assert_close(compute_tree_advantage(rewards, parent), rtr.compute_tree_advantage(rewards, parent))
    tb = TreeRolloutBatch(tokens, mask, old, ref, rewards, parent)
    o, _ = tree_grpo_loss(logits, tb, cfg=GRPOConfig())
    t_, _ = rtr.tree_grpo_loss(logits, rtr.TreeRolloutBatch(tokens, mask, old, ref, rewards, parent),
                               cfg=rg.GRPOConfig())
    torch.testing.assert_close(o, t_, rtol=1e-5, atol=1e-6)
    from saint_llm_posttraining import tree_grpo_trainer as rtt

    assert torch.equal(tree_dynamic_sampling_mask(rewards, parent), rtt.tree_dynamic_sampling_mask(rewards, parent))


@pytest.mark.parametrize("mode", ["mean", "weighted", "max"])
def test_opd_matches_reference(ref_pkgs, mode):
    from saint_llm_posttraining import opd as ro

    gen = torch.Generator().manual_seed(2)
    teachers = [torch.randn(2, 5, 11, generator=gen) for _ in range(3)]
    w = torch.tensor([0.2, 0.5, 0.3]) if mode == "weighted" else None
    a = aggregate_teacher_logits(teachers, weights=w, mode=mode)
    b = ro.aggregate_teacher_logits(teachers, weights=w, mode=mode)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    s = torch.randn(2, 5, 11, generator=gen)
    m = torch.tensor([[0, 1, 1, 1, 0], [1, 1, 0, 0, 0]])
    la, na = opd_kl_loss(s, a, m, temperature=2.0, chunk_rows=3)
    lb, nb = ro.opd_kl_loss(s, b, m, temperature=2.0)
    torch.testing.assert_close(la, lb, rtol=1e-5, atol=1e-6)
    assert na == nb == 5
    assert OPDConfig().aggregation == "mean"


def test_rewards_critique_prm():
    assert unigram_overlap_reward("", "a small cat", target="the small cat") == pytest.approx(2 / 3)
    assert length_target_reward("", "a b c", target_min=5, target_max=8, decay_tokens=4) == pytest.approx(0.5)
    reqs = collect_critique_requests(rewards=torch.tensor([1.0, 0.2, 0.9]), prompts=["a", "b", "c"],
                                     completions=["x", "y", "z"], threshold=0.5)
    assert [(r.rollout_idx, r.original_prompt) for r in reqs] == [(1, "b")]
    toks = torch.tensor([[1, 9, 2, 9, 9], [3, 4, 5, 6, 7]])
    pos = find_step_boundaries(toks, 9)
    assert pos.tolist() == [[1, 3, 4, -1, -1], [-1] * 5]
    head = StepRewardHead(ThinkPRMConfig(hidden_dim=8))
    from saint_llm_b200.posttrain.think_prm import gather_step_scores

    probs, valid = gather_step_scores(torch.randn(2, 5, 8), head, pos)
    assert valid.sum() == 3 and bool((probs[~valid] == 0).all())


@pytest.fixture(scope="module")
def tiny():
    torch.manual_seed(0)
    return SaintLLM(ModelConfig.tiny())


def test_policy_logprobs_and_sft_loss_match_logits_path(tiny):
    tokens = torch.randint(0, 512, (2, 16))
    lp = policy_token_logprobs(tiny, tokens)
    from saint_llm_b200.posttrain import gather_token_logprobs

    torch.testing.assert_close(lp, gather_token_logprobs(tiny(tokens)["logits"], tokens))
    mask = torch.zeros(2, 16, dtype=torch.long)
    mask[:, 8:] = 1
    from saint_llm_b200.posttrain import SFTPackedBatch

    b = SFTPackedBatch(tokens, mask, torch.zeros_like(tokens))
    torch.testing.assert_close(sft_loss(tiny, tokens, mask), sft_cross_entropy(tiny(tokens), b), rtol=1e-5, atol=1e-5)


def test_sft_packing_matches_reference(ref_pkgs):
    from saint_llm_data.tokenizer import CharTokenizer as RT
    from saint_llm_posttraining import sft as rs

    ex = [SFTExample("hi", "there", "sys"), SFTExample("q", "answer"), SFTExample("x", "y")]
    ours = list(pack_sft_into_batch(ex, CharTokenizer(), batch_size=2, seq_len=6, drop_last=False))
    theirs = list(rs.pack_sft_into_batch([rs.SFTExample(e.prompt, e.response, e.system) for e in ex], RT(),
                                         batch_size=2, seq_len=6, drop_last=False))
    assert len(ours) == len(theirs)
    for a, b in zip(ours, theirs, strict=True):
        assert torch.equal(a.tokens, b.tokens) and torch.equal(a.loss_mask, b.loss_mask)
        assert torch.equal(a.segment_ids, b.segment_ids)


def test_rollouts_train_step_and_grm(tiny):
    prompts = torch.randint(0, 512, (2, 6))
    cfg = RolloutGenConfig(group_size=3, max_new_tokens=5, seed=0, eos_token=7)
    tokens, mask = generate_grpo_rollouts(tiny.eval(), prompts, cfg)
    assert tokens.shape == (6, 11) and bool((mask[:, :6] == 0).all())
    assert torch.equal(tokens[:3, :6], prompts[0].expand(3, 6))
    texts = decode_rollouts_for_reward(tokens, lambda ids: ",".join(map(str, ids)), prompt_len=6)
    assert len(texts) == 6
    rewards = torch.tensor([1.0, 0.0, 0.5, 1.0, 1.0, 1.0])
    batch = build_rollout_batch(actor=tiny, ref=None, tokens=tokens, response_mask=mask, rewards=rewards)
    assert torch.equal(batch.old_logprobs, batch.ref_logprobs)
    opt = torch.optim.SGD(tiny.parameters(), lr=1e-3)
    step = grpo_train_step(actor=tiny, optimizer=opt, batch=batch, cfg=GRPOConfig(group_size=3))
    assert step.n_kept_groups == 1 and torch.isfinite(step.loss)
    gcfg = binary_grm_config(good_token_id=5, bad_token_id=6)
    score = judge_completion(tiny.eval(), prompts, gcfg)
    assert score.shape == (2,) and bool(((score >= 0) & (score <= 1)).all())


def test_specialist_pipeline(tiny):
    tok = CharTokenizer(base_vocab=16, unicode_max=512 - 16)
    opt = torch.optim.SGD(tiny.parameters(), lr=1e-4)
    sp = SpecialistPipeline(actor=tiny, ref=None, optimizer=opt, encode=tok.encode, decode=tok.decode,
                            eos_token=tok.eos_token_id)
    out = sp.rl_step(["ab", "cd"], reward_fn=lambda p, c: float(len(c) % 2), cfg=GRPOConfig(group_size=2),
                     rollout_cfg=RolloutGenConfig(group_size=2, max_new_tokens=3, seed=1))
    assert out.n_rollouts == 4
    batch = next(iter(pack_sft_into_batch([SFTExample("ab", "cd")] * 4, tok, batch_size=2, seq_len=8)))
    assert torch.isfinite(sp.sft_step(batch).loss)

"""Post-training and sampling contracts on CPU: GRPO advantages and masks, overlong shaping,
token log-probs, tree advantages, entropy weights, sampling filters and parameters, stop
matching, logit-bias helpers and the paged KV manager's tables."""

import math

import pytest
import torch

from saint_llm_b200.infer.logit_bias import apply_logit_bias, forbid_tokens_bias, force_token_bias
from saint_llm_b200.infer.paged_kv import PagedKVManager, PagePool, PoolExhausted, paged_attention
from saint_llm_b200.infer.sampling import (
    SamplingParams,
    apply_repetition_penalty,
    bias_vector,
    filter_top_k,
    filter_top_p,
    next_token,
)
from saint_llm_b200.infer.stop_sequences import StopSequenceMatcher
from saint_llm_b200.posttrain.grpo import (
    compute_group_advantage,
    dynamic_sampling_mask,
    gather_token_logprobs,
    overlong_reward_shape,
)
from saint_llm_b200.posttrain.gtpo import entropy_weight, per_token_entropy
from saint_llm_b200.posttrain.tree_grpo import compute_tree_advantage, tree_dynamic_sampling_mask


# -------------------------------------------------------------------- GRPO
def test_group_advantage_is_zero_mean_unit_scale_per_group():
    r = torch.tensor([1.0, 0.0, 0.0, 1.0, 3.0, 3.0, 3.0, 3.0])
    a = compute_group_advantage(r, group_size=4)
    g = a.view(2, 4)
    assert torch.allclose(g.mean(-1), torch.zeros(2), atol=1e-6)
    assert torch.allclose(g[0].std(unbiased=False), torch.tensor(1.0), atol=1e-4)
    assert torch.equal(g[1], torch.zeros(4))  # equal rewards carry no signal
    ub = compute_group_advantage(r, group_size=4, unbiased=True)  # Dr.GRPO: centred, not scaled
    assert torch.allclose(ub, torch.tensor([0.5, -0.5, -0.5, 0.5, 0, 0, 0, 0]))
    for bad in (0, 3):
        with pytest.raises(ValueError):
            compute_group_advantage(r, group_size=bad)


def test_dynamic_sampling_drops_uniform_groups():
    r = torch.tensor([1.0, 1.0, 0.0, 1.0, 2.0, 2.0])
    assert dynamic_sampling_mask(r, group_size=2).tolist() == [False, False, True, True, False, False]


def test_overlong_shaping_band():
    r = torch.ones(5)
    lens = torch.tensor([10, 80, 90, 95, 100])
    out = overlong_reward_shape(r, lens, max_length=100, band=(0.8, 1.0))
    assert torch.allclose(out, torch.tensor([1.0, 1.0, 0.5, 0.25, 0.0]))
    assert overlong_reward_shape(r, lens, max_length=100, band=None) is r
    with pytest.raises(ValueError, match="band"):
        overlong_reward_shape(r, lens, max_length=100, band=(0.9, 0.5))


def test_gather_token_logprobs_shifts_and_validates():
    torch.manual_seed(0)
    logits = torch.randn(2, 5, 7)
    toks = torch.randint(0, 7, (2, 5))
    lp = gather_token_logprobs(logits, toks)
    assert lp.shape == (2, 5) and torch.equal(lp[:, 0], torch.zeros(2))
    want = torch.log_softmax(logits[:, :-1].float(), -1).gather(-1, toks[:, 1:, None])[..., 0]
    torch.testing.assert_close(lp[:, 1:], want)
    with pytest.raises(ValueError):
        gather_token_logprobs(logits[0], toks[0])
    with pytest.raises(ValueError):
        gather_token_logprobs(logits, toks[:, :4])


def test_tree_advantage_uses_siblings():
    # root 0 with children 1, 2; child 1 with children 3, 4 (parent of a root is -1)
    r = torch.tensor([0.0, 1.0, 0.0, 1.0, 1.0])
    parent = torch.tensor([-1, 0, 0, 1, 1])
    a = compute_tree_advantage(r, parent)
    assert a.shape == r.shape
    assert a[1] > 0 > a[2]            # the better sibling gets the positive advantage
    assert abs(a[3].item()) < 1e-6 and abs(a[4].item()) < 1e-6  # equal siblings: no signal
    m = tree_dynamic_sampling_mask(r, parent)
    assert bool(m[1]) and bool(m[2]) and not bool(m[3]) and not bool(m[4])


def test_entropy_and_entropy_weights():
    logits = torch.tensor([[[0.0, 0.0, 0.0, 0.0], [10.0, 0.0, 0.0, 0.0]]])
    ent = per_token_entropy(logits)
    assert math.isclose(ent[0, 0].item(), math.log(4), rel_tol=1e-5) and ent[0, 1].item() < 0.01
    mask = torch.tensor([[True, True]])
    w = entropy_weight(ent, mask, alpha=1.0)
    assert w.shape == ent.shape and w[0, 0] > w[0, 1]


# ----------------------------------------------------------------- sampling
def test_sampling_params_validation_and_greedy():
    assert SamplingParams().greedy and not SamplingParams(temperature=0.7).greedy
    for kw in ({"temperature": -1.0}, {"top_k": 0}, {"top_p": 0.0}, {"top_p": 1.5}, {"repetition_penalty": 0.0}):
        with pytest.raises(ValueError):
            SamplingParams(**kw).validate()
    SamplingParams(temperature=0.5, top_k=5, top_p=0.9, repetition_penalty=1.1).validate()


def test_filters_keep_the_right_sets():
    x = torch.tensor([[1.0, 5.0, 3.0, 3.0, -2.0]])
    k2 = filter_top_k(x, 2)
    assert torch.isfinite(k2).tolist() == [[False, True, True, True, False]]  # ties at the k-th value stay
    assert torch.isfinite(filter_top_k(x, 99)).all()
    p = filter_top_p(torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]])), 0.6)
    assert torch.isfinite(p).tolist() == [[True, True, False, False]]
    p0 = filter_top_p(torch.tensor([[0.0, 9.0, 0.0]]), 1e-6)
    assert torch.isfinite(p0).tolist() == [[False, True, False]]  # the best token always stays


def test_repetition_penalty_and_bias_vector():
    logits = torch.tensor([[2.0, -2.0, 1.0]])
    out = apply_repetition_penalty(logits, torch.tensor([[0, 1]]), 2.0)
    assert out.tolist() == [[1.0, -4.0, 1.0]]
    assert apply_repetition_penalty(logits, torch.tensor([[0]]), 1.0) is logits
    v = bias_vector({1: 0.5, 99: 3.0, -1: 1.0}, 3)
    assert v.tolist() == [0.0, 0.5, 0.0]
    assert bias_vector(None, 3) is None and bias_vector({}, 3) is None


def test_next_token_greedy_applies_bias_and_penalty():
    logits = torch.tensor([[1.0, 2.0, 0.5]])
    assert next_token(logits, SamplingParams()).view(-1).tolist() == [1]
    forced = next_token(logits, SamplingParams(), bias=bias_vector(force_token_bias(2), 3))
    assert forced.view(-1).tolist() == [2]
    g = torch.Generator().manual_seed(0)
    picks = {int(next_token(logits, SamplingParams(temperature=1.0, top_k=1), generator=g).view(-1)[0])
             for _ in range(20)}
    assert picks == {1}


def test_logit_bias_helpers():
    x = torch.zeros(1, 4)
    y = apply_logit_bias(x, {**force_token_bias(3), **forbid_tokens_bias([0, 1])})
    assert y.argmax(-1).item() == 3 and y[0, 0] < -1e8 and y[0, 1] < -1e8
    assert apply_logit_bias(x, None) is x or torch.equal(apply_logit_bias(x, None), x)


def test_stop_matcher_multi_token_and_sticky():
    m = StopSequenceMatcher([[5, 6], [9], []])
    assert m.sequences == ((5, 6), (9,))
    assert [m.feed(t) for t in (1, 5, 7, 5, 6)] == [False, False, False, False, True]
    assert m.matched_sequence == (5, 6) and m.feed(1)  # stays matched
    m.reset()
    assert not m.matched() and m.feed(9)
    assert not StopSequenceMatcher([]).feed(1)


# ------------------------------------------------------------------ paging
def test_paged_manager_tables_gather_and_release():
    pools = {"k": PagePool(8, 4, 3), "v": PagePool(8, 4, 3)}
    mgr = PagedKVManager(pools, n_layers=1)
    for req, n in (("a", 6), ("b", 1)):
        mgr.admit(req)
        rows = torch.arange(n * 3, dtype=torch.float32).view(n, 3)
        mgr.append(req, 0, "k", rows)
        mgr.append(req, 0, "v", rows + 100)
    with pytest.raises(KeyError):
        mgr.admit("a")
    table, lens = mgr.block_tables(["a", "b"], 0, "k")
    assert lens.tolist() == [6, 1] and table.shape == (2, 2) and table[1, 1].item() == -1
    padded, plen = mgr.gather_padded(["a", "b"], 0, "k")
    assert padded.shape == (2, 6, 3) and plen.tolist() == [6, 1]
    assert torch.equal(padded[0], torch.arange(18, dtype=torch.bfloat16).view(6, 3))
    q = torch.randn(2, 2, 3)
    out = paged_attention(q, pools["k"], pools["v"], table, lens)
    k0 = padded[1, :1].float()
    v0 = mgr.gather_padded(["b"], 0, "v")[0][0, :1].float()
    torch.testing.assert_close(out[1], (torch.softmax(q[1] @ k0.t() / math.sqrt(3), -1) @ v0))
    used = pools["k"].free_pages
    mgr.release("a")
    assert pools["k"].free_pages == used + 2
    with pytest.raises(PoolExhausted):
        PagePool(1, 2, 3).alloc_many(2)


# ---------------------------------------------------------- surrogate loss
def _batch(B=4, T=6, seed=0):
    from saint_llm_b200.posttrain.grpo import RolloutBatch

    g = torch.Generator().manual_seed(seed)
    mask = torch.zeros(B, T, dtype=torch.bool)
    mask[:, 2:] = True
    old = -torch.rand(B, T, generator=g)
    return RolloutBatch(torch.zeros(B, T, dtype=torch.long), mask, old, old.clone(), torch.tensor([1.0, 0.0, 0.5, 0.5]))


def test_surrogate_on_policy_equals_minus_mean_advantage():
    from saint_llm_b200.posttrain.grpo import GRPOConfig, policy_surrogate_loss

    b = _batch()
    adv = torch.tensor([1.0, -1.0, 0.5, 0.0])
    loss, met = policy_surrogate_loss(b.old_logprobs.clone(), b, adv, GRPOConfig(kl_coef=0.0))
    torch.testing.assert_close(loss, -adv.mean())  # ratio 1 everywhere, KL 0
    assert met["clip_frac"].item() == 0.0 and abs(met["ratio_mean"].item() - 1.0) < 1e-6


def test_surrogate_clipping_stops_the_gradient():
    from saint_llm_b200.posttrain.grpo import GRPOConfig, policy_surrogate_loss

    b = _batch()
    adv = torch.tensor([1.0, 1.0, -1.0, -1.0])
    new = (b.old_logprobs + torch.tensor([0.5, 0.0, -0.5, 0.0]).view(4, 1)).requires_grad_(True)
    loss, met = policy_surrogate_loss(new, b, adv, GRPOConfig(kl_coef=0.0))
    loss.backward()
    g = new.grad
    # row 0: ratio e^0.5 > 1.2 with a positive advantage -> clipped, no gradient;
    # row 2: ratio e^-0.5 < 0.8 with a negative advantage -> clipped, no gradient
    assert g[0, 2:].abs().max() == 0 and g[2, 2:].abs().max() == 0
    assert g[1, 2:].abs().min() > 0 and g[3, 2:].abs().min() > 0
    assert g[:, :2].abs().max() == 0  # prompt tokens never get a gradient
    assert abs(met["clip_frac"].item() - 0.5) < 1e-6


def test_surrogate_kl_is_nonnegative_and_zero_at_reference():
    from saint_llm_b200.posttrain.grpo import GRPOConfig, policy_surrogate_loss

    b = _batch()
    zero = torch.zeros(4)
    _, met0 = policy_surrogate_loss(b.ref_logprobs.clone(), b, zero, GRPOConfig())
    assert abs(met0["kl_penalty"].item()) < 1e-7
    _, met1 = policy_surrogate_loss(b.ref_logprobs + 0.3, b, zero, GRPOConfig())
    assert met1["kl_penalty"].item() > 0


def test_clip_higher_bounds_and_sequence_ratio():
    from saint_llm_b200.posttrain.grpo import GRPOConfig, policy_surrogate_loss

    assert GRPOConfig().clip_bounds == (0.8, 1.2)
    assert GRPOConfig(use_clip_higher=True).clip_bounds == (0.8, 1.28)
    b = _batch()
    new = b.old_logprobs + 0.1
    loss_tok, _ = policy_surrogate_loss(new, b, torch.ones(4), GRPOConfig(kl_coef=0.0))
    loss_seq, _ = policy_surrogate_loss(new, b, torch.ones(4), GRPOConfig(kl_coef=0.0,
                                                                           importance_ratio_level="sequence"))
    # a uniform shift of 0.1 gives the same ratio per token and per sequence
    torch.testing.assert_close(loss_tok, loss_seq)

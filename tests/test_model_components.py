"""Model building blocks on CPU: RoPE, masks, sink softmax, MQA attention oracle, routers and
balancing, Sinkhorn, mHC expand / collapse, compressor pooling, config validation and the
assembled model's shapes and determinism."""

import math

import pytest
import torch

from saint_llm_b200.config import MHCConfig, ModelConfig, MoEConfig
from saint_llm_b200.models.attention.common import (
    RMSNorm,
    apply_partial_rope,
    causal_mask,
    rope_tables,
    scaled_dot_product,
    sliding_window_mask,
    softmax_with_sink,
    window_mask_at,
)
from saint_llm_b200.models.mhc import MHC, sinkhorn_knopp
from saint_llm_b200.models.moe import HashRouter, LearnedRouter, sequence_balance_loss


def test_rope_is_a_rotation_and_relative():
    torch.manual_seed(0)
    x = torch.randn(2, 5, 16)
    cos, sin = rope_tables(5, 8)
    y = apply_partial_rope(x, cos, sin, 8)
    assert torch.equal(y[..., :8], x[..., :8])  # only the last rope_dim channels rotate
    torch.testing.assert_close(y.norm(dim=-1), x.norm(dim=-1))  # norm preserved
    # dot products of rotated q, k depend only on the position difference
    q, k = torch.randn(8), torch.randn(8)
    c, s = rope_tables(12, 8)

    def at(v, p):
        return apply_partial_rope(v.view(1, 1, 8), c[p:p + 1], s[p:p + 1], 8).view(8)

    torch.testing.assert_close(at(q, 7) @ at(k, 4), at(q, 5) @ at(k, 2), rtol=1e-5, atol=1e-5)
    assert torch.equal(apply_partial_rope(x, cos, sin, 0), x)
    with pytest.raises(ValueError):
        rope_tables(4, 7)
    with pytest.raises(ValueError):
        apply_partial_rope(x, *rope_tables(5, 32), 32)


def test_masks():
    assert causal_mask(2, 4).tolist() == [[True, True, True, False], [True, True, True, True]]
    w = sliding_window_mask(5, 2)
    assert w.sum().item() == 9 and bool(w[4, 3]) and not bool(w[4, 2]) and not bool(w[1, 2])
    m = window_mask_at(3, 2, 6, 2)
    assert m.tolist() == [[False, False, True, True, False, False], [False, False, False, True, True, False]]


def test_softmax_with_sink_shrinks_mass():
    s = torch.randn(1, 2, 3, 4)
    assert torch.equal(softmax_with_sink(s, None), torch.softmax(s, -1))
    p = softmax_with_sink(s, torch.tensor([0.0, 50.0]))
    assert torch.all(p[0, 0].sum(-1) < 1) and torch.all(p[0, 1].sum(-1) < 1e-10)
    want = torch.exp(s[0, 0]) / (torch.exp(s[0, 0]).sum(-1, keepdim=True) + 1.0)
    torch.testing.assert_close(p[0, 0], want)


def test_mqa_oracle_equals_broadcast_attention():
    torch.manual_seed(1)
    q = torch.randn(2, 4, 5, 8)
    k, v = torch.randn(2, 1, 7, 8), torch.randn(2, 1, 7, 8)
    mask = causal_mask(5, 7)
    got = scaled_dot_product(q, k, v, mask=mask)
    s = (q @ k.expand(2, 4, 7, 8).transpose(-1, -2)) / math.sqrt(8)
    want = torch.softmax(s.masked_fill(~mask, float("-inf")), -1) @ v.expand(2, 4, 7, 8)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_rmsnorm_cpu():
    n = RMSNorm(6)
    x = torch.randn(3, 6) * 5
    y = n(x)
    torch.testing.assert_close(y.pow(2).mean(-1), torch.ones(3), rtol=1e-4, atol=1e-4)


def test_hash_router_is_deterministic_distinct_and_uniform():
    ids = torch.arange(5000)
    idx, gate = HashRouter.route(ids, 16, 4)
    assert idx.shape == (5000, 4) and torch.equal(idx, HashRouter.route(ids, 16, 4)[0])
    assert (idx >= 0).all() and (idx < 16).all()
    assert all(len(set(r)) == 4 for r in idx[:200].tolist())  # no expert twice per token
    assert torch.allclose(gate, torch.full_like(gate, 0.25))
    counts = torch.bincount(idx.reshape(-1), minlength=16).float()
    assert counts.min() > 0.7 * counts.mean()


def test_learned_router_gates_and_bias_update():
    torch.manual_seed(2)
    cfg = MoEConfig(routed_experts=8, experts_per_token=2)
    r = LearnedRouter(16, 8, 2, cfg, enable_modality_bias=False)
    x = torch.randn(4, 10, 16)
    idx, gate, aff = r(x)
    assert idx.shape == (4, 10, 2) and torch.allclose(gate.sum(-1), torch.ones(4, 10))
    assert (aff > 0).all()
    # the aux-free bias steers selection toward under-loaded experts and never into the gates
    counts = torch.tensor([100.0, 0, 0, 0, 0, 0, 0, 0])
    r.update_bias(counts)
    assert r.aux_free_bias[0] < 0 and (r.aux_free_bias[1:] > 0).all()
    r.aux_free_bias[3] = 100.0
    idx2, gate2, _ = r(x)
    assert (idx2 == 3).any(-1).all()
    torch.testing.assert_close(gate2.sum(-1), torch.ones(4, 10))
    loss = sequence_balance_loss(aff, idx)
    assert loss.ndim == 0 and loss > 0


def test_sinkhorn_converges_to_doubly_stochastic():
    torch.manual_seed(3)
    p = sinkhorn_knopp(torch.randn(5, 4, 4) * 3, 50)
    torch.testing.assert_close(p.sum(-1), torch.ones(5, 4), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(p.sum(-2), torch.ones(5, 4), rtol=1e-3, atol=1e-3)
    assert (p >= 0).all()


def test_mhc_expand_collapse_and_identity_start():
    x = torch.randn(2, 3, 8)
    e = MHC.expand(x, 4)
    assert e.shape == (2, 3, 4, 8)
    torch.testing.assert_close(MHC.collapse(e), x)  # the streams start as copies; collapse averages
    m = MHC(8, MHCConfig(expansion_factor=2, sinkhorn_iters=10))
    inner, a, b, c = m.split(torch.randn(2, 3, 2, 8))
    assert inner.shape == (2, 3, 8) and a.shape == (2, 3, 2) and b.shape == (2, 3, 2, 2) and c.shape == (2, 3, 2)
    torch.testing.assert_close(b.sum(-1), torch.ones(2, 3, 2), rtol=1e-2, atol=1e-2)


def test_compressor_pool_is_a_convex_combination():
    from saint_llm_b200.models.attention.csa import TokenLevelCompressor

    torch.manual_seed(4)
    comp = TokenLevelCompressor(16, 8, 4)
    with torch.no_grad():
        comp.bias_b.normal_()
    c = torch.randn(2, 12, 8)
    z = torch.randn(2, 12, 8)
    out = comp.pool(c, z)
    assert out.shape == (2, 3, 8)
    cb = c.view(2, 3, 4, 8)
    assert (out <= cb.amax(2) + 1e-5).all() and (out >= cb.amin(2) - 1e-5).all()
    assert comp(torch.randn(2, 3, 16)).shape == (2, 0, 8)  # fewer tokens than one block


def test_config_is_frozen_and_strict():
    with pytest.raises(ValueError):  # unknown fields are rejected (the checkpoint schema is fixed)
        ModelConfig.model_validate({**ModelConfig.tiny().model_dump(), "no_such_field": 1})
    with pytest.raises(Exception):  # frozen
        ModelConfig.tiny().hidden_dim = 3  # type: ignore[misc]
    again = ModelConfig.model_validate(ModelConfig.tiny().model_dump())
    assert again == ModelConfig.tiny()


def test_model_forward_shapes_and_determinism():
    from saint_llm_b200.models import SaintLLM

    cfg = ModelConfig.tiny()
    torch.manual_seed(0)
    a = SaintLLM(cfg)
    torch.manual_seed(0)
    b = SaintLLM(cfg)
    ids = torch.randint(0, cfg.vocab_size, (2, 24))
    out_a, out_b = a(ids), b(ids)
    assert out_a["logits"].shape == (2, 24, cfg.vocab_size)
    assert torch.equal(out_a["logits"], out_b["logits"])  # seeded init is reproducible
    assert torch.isfinite(out_a["logits"]).all()

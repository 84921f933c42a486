"""Model options on CPU: activation checkpointing, where linear quantisation applies, the
reasoning-effort head, the video tokenizer stand-in and the small_flash preset."""

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from saint_llm_b200.config import ModelConfig
from saint_llm_b200.models import SaintLLM
from saint_llm_b200.models.linear import Fp4Linear, Fp8Linear


def _ce(model, ids):
    out = model(ids)
    loss = F.cross_entropy(out["logits"][:, :-1].reshape(-1, model.cfg.vocab_size), ids[:, 1:].reshape(-1))
    aux = out.get("aux_loss")
    return loss + (0.01 * aux if isinstance(aux, torch.Tensor) else 0.0)


# ------------------------------------------------------------- activation checkpointing
def test_activation_checkpointing_changes_nothing_but_memory():
    cfg = ModelConfig.tiny()
    assert cfg.activation_checkpointing is False
    torch.manual_seed(0)
    off = SaintLLM(cfg).train()
    on = SaintLLM(cfg.model_copy(update={"activation_checkpointing": True})).train()
    on.load_state_dict(off.state_dict())
    ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=torch.Generator().manual_seed(1))
    lo, ln = _ce(off, ids), _ce(on, ids)
    torch.testing.assert_close(lo, ln)
    lo.backward()
    ln.backward()
    g_on = dict(on.named_parameters())
    n = 0
    for name, p in off.named_parameters():
        if p.grad is None:
            assert g_on[name].grad is None or not g_on[name].grad.any(), name
            continue
        torch.testing.assert_close(g_on[name].grad, p.grad, atol=1e-6, rtol=1e-4, msg=name)
        n += 1
    assert n > 50
    with torch.no_grad():  # eval / no-grad forwards never checkpoint and stay finite
        assert torch.isfinite(on.eval()(ids)["logits"]).all()


# ------------------------------------------------------------- where quantisation applies
@pytest.mark.parametrize("mode,cls", [("fp8", Fp8Linear), ("fp4", Fp4Linear)])
def test_linear_quant_reaches_projections_but_not_router_indexer_or_head(mode, cls):
    cfg = ModelConfig.tiny().model_copy(update={"linear_quant": mode})
    torch.manual_seed(0)
    m = SaintLLM(cfg)
    csa = next(b.attention for b in m.blocks if type(b.attention).__name__ == "CSA")
    assert isinstance(csa.q_compressor, cls) and isinstance(csa.q_up, cls) and isinstance(csa.k_proj, cls)
    assert isinstance(csa.output.final_proj, cls) and all(isinstance(g, cls) for g in csa.output.group_projs)
    assert isinstance(csa.kv_compressor.w_b_kv, cls)
    # the indexer (its own compressor included) and the router score projection stay plain
    assert not any(isinstance(x, (Fp8Linear, Fp4Linear)) for x in csa.indexer.modules())
    moe = m.blocks[-1].moe
    assert moe.router is not None and type(moe.router.score_proj) is nn.Linear
    assert any(isinstance(x, cls) for x in moe.shared_experts.modules())
    assert not isinstance(m.lm_head, (Fp8Linear, Fp4Linear))
    ids = torch.randint(0, cfg.vocab_size, (1, 16), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        assert torch.isfinite(m(ids)["logits"]).all()
    with pytest.raises(ValueError):
        from saint_llm_b200.models.linear import make_linear_factory

        make_linear_factory("int4")  # type: ignore[arg-type]


# ------------------------------------------------------------------ reasoning effort head
def test_effort_router_contract():
    from saint_llm_b200.models.multimodal import (EFFORT_TIER_NAMES, EffortConfig, EffortRouter,
                                                  effort_id_to_token, effort_tier_to_id)

    cfg = EffortConfig()
    assert (cfg.n_tiers, cfg.hidden, cfg.enabled) == (5, 64, False)
    head = EffortRouter(32, cfg)
    pooled = torch.randn(3, 32)
    tier = torch.tensor([0, 2, 4])
    out = head(pooled, tier)
    assert out["budget"].shape == (3,) and not out["budget"].any() and not out["terminate_logit"].any()
    with pytest.raises(ValueError):
        head(pooled, torch.tensor([0, 5, 1]))
    with pytest.raises(ValueError):
        head(pooled, tier.view(3, 1))
    # once the zero init is perturbed, tiers are distinguishable and budgets stay >= 0
    with torch.no_grad():
        for p in head.parameters():
            p.normal_(0, 0.5)
    same = torch.randn(1, 32).expand(5, 32)
    out = head(same, torch.arange(5))
    assert (out["budget"] >= 0).all() and out["terminate_logit"].unique().numel() > 1
    out["terminate_logit"].sum().backward()
    assert head.tier_emb.weight.grad is not None and head.tier_emb.weight.grad.abs().sum() > 0
    assert EFFORT_TIER_NAMES == ("low", "medium", "high", "xhigh", "max")
    assert [effort_tier_to_id(n.upper()) for n in EFFORT_TIER_NAMES] == [0, 1, 2, 3, 4]
    assert effort_id_to_token(3) == "<|effort:3|>"
    for bad in (lambda: effort_tier_to_id("extreme"), lambda: effort_id_to_token(5), lambda: effort_id_to_token(-1)):
        with pytest.raises(ValueError):
            bad()


# ------------------------------------------------------------------------ video stand-in
def test_fake_video_tokenizer():
    from saint_llm_b200.models.multimodal import FakeVideoTokenizer, encode_video_clips

    tok = FakeVideoTokenizer(vision_dim=16, patches_per_frame=3, seed=1)
    assert (tok.vision_dim, tok.patches_per_frame) == (16, 3)
    clip = torch.rand(4, 3, 8, 8)
    feats = tok.encode(clip)
    assert feats.shape == (12, 16)
    torch.testing.assert_close(feats, FakeVideoTokenizer(vision_dim=16, patches_per_frame=3, seed=1).encode(clip))
    assert not torch.allclose(feats, FakeVideoTokenizer(vision_dim=16, patches_per_frame=3, seed=2).encode(clip))
    assert not torch.equal(feats[0], feats[1])  # patches of one frame differ
    for bad in (torch.rand(3, 8, 8), torch.rand(2, 4, 8, 8)):
        with pytest.raises(ValueError):
            tok.encode(bad)
    with pytest.raises(ValueError):
        FakeVideoTokenizer(vision_dim=0, patches_per_frame=3)
    out = encode_video_clips([clip, clip[:2]], tok)
    assert [o.shape[0] for o in out] == [12, 6]


# ------------------------------------------------------------------------ small_flash
def test_small_flash_preset():
    cfg = ModelConfig.small_flash()
    for dim in (cfg.hidden_dim, cfg.attention.query_compression_dim, cfg.attention.query_heads * cfg.attention.head_dim,
                cfg.moe.expert_intermediate_dim):
        assert dim % 32 == 0  # every FP4-quantised input width is a whole number of 32-blocks
    with torch.device("meta"):
        m = SaintLLM(cfg)
    total = sum(p.numel() for p in m.parameters())
    assert 80_000_000 <= total <= 300_000_000, total

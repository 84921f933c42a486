"""Native single-token decode attention (one kernel per layer) against the eager
composition of the same step, for SWA, HCA and CSA layers with random caches."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fill(st, gen):
    for t in [st.k, st.v] + ([st.kv.cb, st.kv.zb, st.kv.entries] if st.kv is not None else []) + \
             ([st.idx.cb, st.idx.zb, st.idx.entries] if st.idx is not None else []):
        t.copy_(torch.randn(t.shape, generator=gen).to(t.device, t.dtype))


def _state(st):
    ts = [st.k, st.v]
    for r in (st.kv, st.idx):
        if r is not None:
            ts += [r.cb, r.zb, r.entries]
    return ts


@pytest.mark.parametrize("pos_val", [3, 130, 517])
def test_decode_attention_matches_eager(cuda, pos_val):
    from saint_llm_b200.config import AttentionConfig, CSAConfig, ModelConfig
    from saint_llm_b200.infer.static_decode import StaticDecoder, _attend_layer, _attend_layer_eager
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.models.attention.common import rope_tables

    base = ModelConfig.tiny()
    att = AttentionConfig(**{**base.attention.model_dump(), "query_heads": 8, "head_dim": 128})
    csa = CSAConfig(**{**base.csa.model_dump(), "attention_top_k": 16})
    cfg = base.model_copy(update={"attention": att, "csa": csa, "n_layers": 4})
    torch.manual_seed(0)
    model = SaintLLM(cfg).to(cuda).to(torch.bfloat16).eval()
    with torch.no_grad():
        for blk in model.blocks:
            if blk.attention.sink_logit is not None:
                blk.attention.sink_logit.normal_()
    dec = StaticDecoder(model, 3, 640)
    gen = torch.Generator().manual_seed(1)
    pos = torch.tensor(pos_val, dtype=torch.long, device=cuda)
    cos, sin = rope_tables(640, cfg.attention.rope_dim, cfg.attention.rope_theta, cuda)
    cos, sin = cos[pos_val:pos_val + 1], sin[pos_val:pos_val + 1]
    kinds = set()
    with torch.no_grad():
        for st in dec.layers:
            kinds.add(type(st.attn).__name__)
            _fill(st, gen)
            h = torch.randn(3, 1, cfg.hidden_dim, generator=gen).to(cuda, torch.bfloat16)
            saved = [t.clone() for t in _state(st)]
            got = _attend_layer(st, h, pos, cos, sin)
            after_native = [t.clone() for t in _state(st)]
            for t, s in zip(_state(st), saved, strict=True):
                t.copy_(s)
            want = _attend_layer_eager(st, h, pos, cos, sin)
            torch.cuda.synchronize()
            for a, b in zip(after_native, _state(st), strict=True):
                assert torch.equal(a, b)  # identical cache updates
            err = (got.float() - want.float()).abs().max().item()
            assert err <= 3e-2 * want.float().abs().max().item() + 1e-3, (type(st.attn).__name__, err)
    assert {"CSA", "HCA"} <= kinds

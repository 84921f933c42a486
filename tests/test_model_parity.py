"""Eager model vs the unmodified reference package (CPU, fp32)."""

import pytest
import torch


def _pair(ref_pkgs, update=None, preset="tiny"):
    from saint_llm_core.config import ModelConfig as RC
    from saint_llm_core.model import SaintLLM as RM

    from saint_llm_b200.config import ModelConfig as OC
    from saint_llm_b200.models import SaintLLM as OM

    rc, oc = getattr(RC, preset)(), getattr(OC, preset)()
    if update:
        rc, oc = rc.model_copy(update=update), oc.model_copy(update=update)
    torch.manual_seed(0)
    r = RM(rc)
    torch.manual_seed(0)
    o = OM(oc)
    return r, o


@pytest.mark.parametrize("update", [None, {"moe_use_grouped_gemm": True},
                                    {"n_sink_tokens": 2, "final_logit_softcap": 30.0},
                                    {"init_scheme": "umup"},
                                    {"linear_quant": "fp8"}, {"linear_quant": "fp4"}])
def test_same_init_and_outputs(ref_pkgs, update):
    r, o = _pair(ref_pkgs, update)
    rs, os_ = r.state_dict(), o.state_dict()
    assert list(rs) == list(os_)
    for k in rs:
        assert rs[k].shape == os_[k].shape, k
        assert torch.equal(rs[k], os_[k]), f"init differs at {k}"
    x = torch.randint(0, r.cfg.vocab_size, (2, 37))
    ro, oo = r(x), o(x)
    torch.testing.assert_close(oo["logits"], ro["logits"], atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(oo["mtp_logits"][0], ro["mtp_logits"][0], atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(oo["aux_loss"], ro["aux_loss"], atol=1e-5, rtol=1e-4)
    (ro["logits"].square().mean() + ro["mtp_logits"][0].mean()).backward()
    (oo["logits"].square().mean() + oo["mtp_logits"][0].mean()).backward()
    for (n, rp), (_, op) in zip(r.named_parameters(), o.named_parameters()):
        if rp.grad is None:
            assert op.grad is None or float(op.grad.abs().max()) == 0.0, n
            continue
        torch.testing.assert_close(op.grad, rp.grad, atol=1e-5, rtol=1e-3, msg=n)


def test_checkpoint_cross_load(ref_pkgs, tmp_path):
    from saint_llm_training.checkpoint import load_checkpoint as rload
    from saint_llm_training.checkpoint import save_checkpoint as rsave

    from saint_llm_b200.train import load_checkpoint, save_checkpoint

    r, o = _pair(ref_pkgs)
    torch.manual_seed(3)
    for p in r.parameters():
        p.data.add_(torch.randn_like(p) * 0.01)
    rsave(tmp_path / "ref.pt", r, step=7, extra={"a": 1})
    meta = load_checkpoint(tmp_path / "ref.pt", o)
    assert meta["step"] == 7 and meta["extra"] == {"a": 1}
    for (k, v), (_, w) in zip(r.state_dict().items(), o.state_dict().items()):
        assert torch.equal(v, w), k
    save_checkpoint(tmp_path / "ours.pt", o, step=9)
    r2, _ = _pair(ref_pkgs)
    assert rload(tmp_path / "ours.pt", r2)["step"] == 9

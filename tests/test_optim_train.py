"""Optimizer, losses, trainer, schedule and checkpoint behaviour (CPU)."""

import math

import pytest
import torch
from torch import nn


def test_newton_schulz_parity(ref_pkgs):
    from saint_llm_optim.newton_schulz import hybrid_newton_schulz as ref_ns

    from saint_llm_b200.optim.newton_schulz import batched_newton_schulz, hybrid_newton_schulz

    torch.manual_seed(0)
    for shape in [(64, 32), (32, 64), (48, 48)]:
        g = torch.randn(*shape)
        torch.testing.assert_close(hybrid_newton_schulz(g), ref_ns(g))
        torch.testing.assert_close(batched_newton_schulz(g[None], precision="fp32")[0], ref_ns(g),
                                   atol=2e-4, rtol=1e-3)


def test_muon_matches_reference(ref_pkgs):
    from saint_llm_optim.muon import Muon as RefMuon

    from saint_llm_b200.optim import Muon

    torch.manual_seed(0)
    w0 = torch.randn(32, 16)
    a, b = nn.Parameter(w0.clone()), nn.Parameter(w0.clone())
    oa, ob = Muon([a], lr=0.02), RefMuon([b], lr=0.02)
    for _ in range(3):
        g = torch.randn(32, 16)
        a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    torch.testing.assert_close(a, b)
    torch.testing.assert_close(oa.state[a]["momentum_buffer"], ob.state[b]["momentum_buffer"])


def test_muon_main_grad_and_3d():
    from saint_llm_b200.optim import Muon

    p = nn.Parameter(torch.randn(3, 8, 4))
    p.main_grad = torch.randn(3, 8, 4)
    before = p.detach().clone()
    Muon([p]).step()
    assert not torch.equal(before, p.detach())
    q = nn.Parameter(torch.randn(3, 8, 4))
    q.grad = torch.randn(3, 8, 4)
    with pytest.raises(ValueError):
        Muon([q], strict_2d=True).step()


def test_qk_clip_device_buffer():
    from saint_llm_b200.config import AttentionConfig
    from saint_llm_b200.models.attention import SWAttention
    from saint_llm_b200.optim import Muon

    layer = SWAttention(32, AttentionConfig(query_heads=2, head_dim=16, query_compression_dim=16,
                                            output_proj_groups=1, attention_intermediate_dim=16, rope_dim=8))
    before = layer.q_up.weight.detach().clone()
    opt = Muon([nn.Parameter(torch.zeros(2, 2))], qk_clip_tau=100.0, qk_clip_layers=[layer])
    layer.max_attn_logit.fill_(400.0)
    opt.step()
    torch.testing.assert_close(layer.q_up.weight, before * 0.5)
    assert list(opt.qk_clip_count.values()) == [1]
    layer.max_attn_logit.fill_(50.0)
    opt.step()
    assert list(opt.qk_clip_count.values()) == [1]


def test_param_split_matches_reference(ref_pkgs):
    from saint_llm_core.config import ModelConfig as RC
    from saint_llm_core.model import SaintLLM as RM
    from saint_llm_optim.param_groups import split_for_muon_adamw as rsplit

    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import split_for_muon_adamw

    torch.manual_seed(0)
    rm, ra = rsplit(RM(RC.tiny()))
    om, oa = split_for_muon_adamw(SaintLLM(ModelConfig.tiny()))
    assert [p.shape for p in rm] == [p.shape for p in om]
    assert [p.shape for p in ra] == [p.shape for p in oa]


def test_losses_match_reference(ref_pkgs):
    from saint_llm_core.config import ModelConfig as RC
    from saint_llm_training.losses import make_loss_fn as rmake

    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.train import make_loss_fn

    torch.manual_seed(0)
    cfg = ModelConfig.tiny()
    m = SaintLLM(cfg)
    x = torch.randint(0, cfg.vocab_size, (2, 20))
    rc = RC.tiny()
    torch.testing.assert_close(make_loss_fn(cfg.mtp, moe_cfg=cfg.moe)(m, x), rmake(rc.mtp, moe_cfg=rc.moe)(m, x))


def test_trainer_loop_and_skip(tmp_path):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.train import CheckpointRotator, Trainer, make_loss_fn, warmup_cosine_schedule

    torch.manual_seed(0)
    cfg = ModelConfig.tiny()
    m = SaintLLM(cfg)
    mu, ad = split_for_muon_adamw(m)
    opt = MuonAdamW(mu, ad, lr=0.02, adamw_lr=3e-3)
    sched = warmup_cosine_schedule(opt, warmup_steps=1, total_steps=10)
    seen = []
    tr = Trainer(m, opt, loss_fn=make_loss_fn(cfg.mtp, moe_cfg=cfg.moe), lr_scheduler=sched, grad_clip_norm=1.0,
                 metrics_callback=lambda s, d: seen.append((s, d)), gradient_accumulation_steps=2,
                 loss_spike_factor=10.0)
    batch = torch.randint(0, cfg.vocab_size, (2, 16))
    losses = [tr.train_step(batch) for _ in range(8)]
    assert tr.step == 4 and len(seen) == 4
    assert losses[-1] < losses[0]
    tr.loss_fn = lambda model, b: torch.tensor(float("nan"), requires_grad=True)
    tr.train_step(batch)
    assert tr.skipped_steps == 1 and seen[-1][1].get("skip_reason_nan") == 1.0
    rot = CheckpointRotator(tmp_path / "ckpt.pt", keep_last_n=2)
    for s in (1, 2, 3):
        rot.save(tr, step=s)
    assert [p.name for p in rot.saved_paths] == ["ckpt.step2.pt", "ckpt.step3.pt"]
    assert isinstance(tr.load(rot.saved_paths[-1]), dict)


def test_atomic_checkpoint_and_sharded(tmp_path):
    from saint_llm_b200.train import checkpoint as ck

    m = nn.Linear(4, 4)
    ck.save_checkpoint(tmp_path / "a.pt", m, step=3)
    assert not (tmp_path / "a.pt.tmp").exists()
    ck.save_sharded(tmp_path / "sh", m.state_dict(), {"x": 1}, step=5, rank=1, world_size=2)
    ck.save_sharded(tmp_path / "sh", m.state_dict(), {"x": 0}, step=5, rank=0, world_size=2)
    data = ck.load_sharded(tmp_path / "sh")
    assert data["step"] == 5 and [o["x"] for o in data["optim"]] == [0, 1]
    out = ck.sharded_to_v1(tmp_path / "sh", tmp_path / "v1.pt")
    m2 = nn.Linear(4, 4)
    assert ck.load_checkpoint(out, m2)["step"] == 5
    torch.testing.assert_close(m2.weight, m.weight)


def test_expert_layout_converters():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.train import experts_to_per_module, experts_to_stacked

    torch.manual_seed(0)
    per = SaintLLM(ModelConfig.tiny())
    grouped = SaintLLM(ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True}))
    grouped.load_state_dict(experts_to_stacked(per.state_dict()))
    back = experts_to_per_module(grouped.state_dict())
    for k, v in per.state_dict().items():
        torch.testing.assert_close(back[k], v)
    x = torch.randint(0, 512, (1, 12))
    torch.testing.assert_close(per(x)["logits"], grouped(x)["logits"], atol=1e-5, rtol=1e-4)


def test_wandb_logger_prefix():
    from unittest.mock import MagicMock

    from saint_llm_b200.train import WandbLogger

    wb = MagicMock()
    lg = WandbLogger(project="p", wandb_module=wb, mode="disabled")
    lg(3, {"loss": 1.0, "eval/ppl": 2.0})
    wb.log.assert_called_with({"train/loss": 1.0, "eval/ppl": 2.0}, step=3)


def test_schedule_shape():
    from saint_llm_b200.train import warmup_cosine_schedule

    p = nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    s = warmup_cosine_schedule(opt, warmup_steps=2, total_steps=6, min_lr_ratio=0.1)
    lrs = []
    for _ in range(6):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        s.step()
    assert lrs[0] < 1e-6 and math.isclose(max(lrs), 1.0, rel_tol=1e-6)


def test_train_step_api_cpu():
    """TrainStep on CPU (eager path) with main_grad buffers: loss goes down."""
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.train.engine import attach_main_grads
    from saint_llm_b200.train.step import TrainStep

    torch.manual_seed(0)
    cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
    m = SaintLLM(cfg)
    params = attach_main_grads(m)
    mu, ad = split_for_muon_adamw(m)
    step = TrainStep(m, MuonAdamW(mu, ad, lr=0.02, adamw_lr=3e-3), micro_batches=2, params=params)
    tok = torch.randint(0, cfg.vocab_size, (2, 1, 24))
    losses = [step(tok) for _ in range(5)]
    assert losses[-1] < losses[0]


def test_trainer_window_one_host_read_and_skip_rules():
    """``train_window``: a whole accumulation window per call; a non-finite loss anywhere
    in it drops the window; the spike rule needs four accepted step losses first."""
    from saint_llm_b200.train import Trainer
    from saint_llm_b200.train.trainer import SkipRule

    rule = SkipRule(nonfinite=True, spike_factor=2.0, window=8)
    assert rule.reason(float("inf")) == "nan" and rule.reason(1e9) is None  # no history yet
    for v in (1.0, 1.1, 0.9, 1.0):
        rule.accept(v)
    assert rule.reason(2.5) == "spike" and rule.reason(1.5) is None
    codes = rule.reasons_device(torch.tensor([1.0, float("nan"), 3.0]))
    assert codes.tolist() == [0, 1, 2]

    torch.manual_seed(0)
    m = nn.Linear(8, 1)
    opt = torch.optim.SGD(m.parameters(), lr=0.1)
    seen = []

    def loss_fn(model, b):
        return ((model(b.float()) - 1.0) ** 2).mean()

    tr = Trainer(m, opt, loss_fn=loss_fn, gradient_accumulation_steps=2,
                 metrics_callback=lambda s, d: seen.append(d))
    xs = [torch.randn(4, 8) for _ in range(2)]
    w0 = m.weight.detach().clone()
    vals = tr.train_window(xs)
    assert len(vals) == 2 and tr.step == 1 and not torch.equal(w0, m.weight)
    assert "perf/step_s" in seen[-1] or len(seen) == 1
    w1 = m.weight.detach().clone()
    tr.loss_fn = lambda model, b: (model(b.float()).sum() * float("nan"))
    tr.train_window(xs)
    assert tr.skipped_steps == 1 and tr.step == 1 and torch.equal(w1, m.weight)
    assert seen[-1].get("skip_reason_nan") == 1.0
    with pytest.raises(ValueError):
        tr.train_window(xs[:1])
    with pytest.raises(ValueError, match="grad_clip_norm"):
        Trainer(m, opt, loss_fn=loss_fn, grad_clip_norm=0.0)


def test_build_training_consumes_run_config():
    """``build_training``: a CPU job from ModelConfig + RunConfig steps and learns; fields
    this builder cannot honour raise instead of being ignored."""
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.train.launch import build_training

    cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
    run = RunConfig(grad_accum=2, micro_batch=1, seq_len=16, lr=0.02, adamw_lr=3e-3, seed=3,
                    param_dtype="float32", compute_dtype="float32")
    job = build_training(cfg, run, torch.device("cpu"))
    torch.manual_seed(0)
    batch = torch.randint(0, cfg.vocab_size, (2, 1, 16))
    losses = [job.step(batch) for _ in range(4)]
    assert losses[-1] < losses[0]
    assert job.optimizer.param_groups[0]["lr"] == 0.02
    for bad in ({"tp": 2}, {"grad_dtype": "bfloat16"}, {"zero": "fsdp"}):
        with pytest.raises(ValueError):
            build_training(cfg, run.model_copy(update=bad), torch.device("cpu"))


def test_init_state_preallocates_without_changing_the_update():
    """``MuonAdamW.init_state`` creates exactly the buffers the first step would (so a graph
    capture can plan memory with them) and the updates stay identical; ``param_filter``
    excludes parameters another rank owns."""
    from saint_llm_b200.optim import MuonAdamW

    torch.manual_seed(0)
    mats = [nn.Parameter(torch.randn(16, 8)) for _ in range(3)]
    vecs = [nn.Parameter(torch.randn(8)) for _ in range(2)]
    grads = [torch.randn_like(p) for p in mats + vecs]

    def run(pre: bool, flt=None):
        ps = [nn.Parameter(p.detach().clone()) for p in mats + vecs]
        opt = MuonAdamW(ps[:3], ps[3:], lr=0.01, qk_clip_enabled=False, ns_impl="torch")
        opt.param_filter = flt
        if pre:
            n = opt.init_state()
            assert n > 0
        for p, g in zip(ps, grads, strict=True):
            p.grad = g.clone()
        opt.step()
        return ps, opt

    a, _ = run(False)
    b, opt_b = run(True)
    for x, y in zip(a, b, strict=True):
        assert torch.equal(x, y)
    assert len(opt_b.state) == 5
    _, opt_c = run(True, flt=lambda p: p.dim() == 1)  # this rank owns only the vectors
    assert len(opt_c.state) == 2 and all(p.dim() == 1 for p in opt_c.state)

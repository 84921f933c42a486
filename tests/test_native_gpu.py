"""Native sm_100a kernels vs the fp32 eager PyTorch oracle of the same op (GPU)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(x, y):
    return ((x.float() - y.float()).norm() / (y.float().norm() + 1e-12)).item()


def _bf(t):
    return t.to(torch.bfloat16).float()


def test_rmsnorm_native(cuda):
    from saint_llm_b200.models.attention.common import RMSNorm
    from saint_llm_b200.ops import backend

    torch.manual_seed(0)
    m = RMSNorm(2048).to(cuda)
    m.weight.data.uniform_(0.5, 1.5)
    x = torch.randn(300, 2048, device=cuda, requires_grad=True)
    g = torch.randn(300, 2048, device=cuda)
    with backend.eager_mode():
        m(x).backward(g)
    gx0, gw0 = x.grad.clone(), m.weight.grad.clone()
    with backend.eager_mode():
        y0 = m(x)
    x.grad = None
    m.weight.grad = None
    y1 = m(x)
    y1.backward(g.to(y1.dtype))
    assert _rel(y1, y0) < 1e-2
    assert _rel(x.grad, gx0) < 2e-2
    assert _rel(m.weight.grad, gw0) < 1e-2


@pytest.mark.parametrize("norm_first", [False, True])
def test_rope_norm_native(cuda, norm_first):
    from saint_llm_b200.models.attention.common import apply_partial_rope, rope_tables
    from saint_llm_b200.ops.norm import rope_norm

    torch.manual_seed(0)
    T, H, d, rd = 64, 4, 128, 64
    x = torch.randn(T, H, d, device=cuda, requires_grad=True)
    w = (torch.rand(d, device=cuda) + 0.5).requires_grad_(True)
    cos, sin = rope_tables(T, rd, 10000.0, cuda)

    def ref(x, w):
        xt = x.transpose(0, 1)

        def norm(z):
            return w * z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + 1e-6)
        y = apply_partial_rope(norm(xt), cos, sin, rd) if norm_first else norm(apply_partial_rope(xt, cos, sin, rd))
        return y.transpose(0, 1)

    g = torch.randn(T, H, d, device=cuda)
    y0 = ref(x, w)
    y0.backward(g)
    gx0, gw0 = x.grad.clone(), w.grad.clone()
    x.grad = None
    w.grad = None
    y1 = rope_norm(x, w, cos, sin, rd, norm_first=norm_first)
    y1.backward(g.to(y1.dtype))
    assert _rel(y1, y0) < 1e-2
    assert _rel(x.grad, gx0) < 2e-2
    assert _rel(w.grad, gw0) < 2e-2


def test_mhc_native(cuda):
    from saint_llm_b200.config import MHCConfig
    from saint_llm_b200.models.mhc import MHC
    from saint_llm_b200.ops import backend

    torch.manual_seed(0)
    n, d = 4, 256
    m = MHC(d, MHCConfig(expansion_factor=n, sinkhorn_iters=20)).to(cuda)
    with torch.no_grad():
        for w in (m.w_pre, m.w_res, m.w_post):
            w.weight.normal_(0, 0.02)
        m.norm.weight.uniform_(0.5, 1.5)
        for p in (m.alpha_pre, m.alpha_res, m.alpha_post):
            p.fill_(0.5)
        m.s_res.normal_(0, 0.3)
    x = torch.randn(2, 70, n, d, device=cuda, requires_grad=True)
    inner_w = torch.randn(d, d, device=cuda) / d ** 0.5
    g = torch.randn(2, 70, n, d, device=cuda)

    def run():
        inner, a, b, c = m.split(x)
        out = m.combine(x, torch.tanh(inner.float() @ inner_w), b, c)
        out.float().backward(g)
        return out

    with backend.eager_mode():
        y0 = run()
    grads0 = {k: p.grad.clone() for k, p in m.named_parameters()}
    gx0 = x.grad.clone()
    m.zero_grad()
    x.grad = None
    y1 = run()
    assert _rel(y1, y0) < 2e-2
    assert _rel(x.grad, gx0) < 3e-2
    for k, p in m.named_parameters():
        assert _rel(p.grad, grads0[k]) < 5e-2, k


def _expert_ref(h, idx, gate, wg, wu, wd, gmax=10.0, lo=-10.0, hi=10.0):
    out = torch.zeros_like(h)
    for e in range(wg.shape[0]):
        tok, slot = (idx == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        x = h[tok]
        y = (F.silu((x @ wg[e].t()).clamp(max=gmax)) * (x @ wu[e].t()).clamp(lo, hi)) @ wd[e].t()
        out = out.index_add(0, tok, gate[tok, slot].unsqueeze(-1) * y)
    return out


@pytest.mark.parametrize("T,E,k,D,I", [(300, 8, 2, 256, 128), (1024, 16, 4, 512, 384)])
def test_routed_experts_fixed_routing(cuda, T, E, k, D, I):
    from saint_llm_b200.ops.moe import GroupedSwiGLUExperts
    from saint_llm_b200.ops.moe_native import routed_experts

    torch.manual_seed(0)
    ex = GroupedSwiGLUExperts(D, I, E).to(cuda)
    with torch.no_grad():
        for w in (ex.gate_weight, ex.up_weight, ex.down_weight):
            w.copy_(_bf(torch.randn_like(w) * 0.05))
    h = _bf(torch.randn(T, D, device=cuda)).requires_grad_(True)
    idx = torch.stack([torch.randperm(E, device=cuda)[:k] for _ in range(T)])
    gate = torch.rand(T, k, device=cuda).requires_grad_(True)
    g = torch.randn(T, D, device=cuda)
    y0 = _expert_ref(h, idx, gate, ex.gate_weight, ex.up_weight, ex.down_weight)
    y0.backward(g)
    ref = {"h": h.grad.clone(), "gate": gate.grad.clone(), "wg": ex.gate_weight.grad.clone(),
           "wu": ex.up_weight.grad.clone(), "wd": ex.down_weight.grad.clone()}
    h.grad = None
    gate.grad = None
    ex.zero_grad()
    y1 = routed_experts(h, idx, gate, ex)
    y1.float().backward(g)
    assert _rel(y1, y0) < 1e-2
    assert _rel(h.grad, ref["h"]) < 2e-2
    assert _rel(gate.grad, ref["gate"]) < 2e-2
    assert _rel(ex.gate_weight.grad, ref["wg"]) < 2e-2
    assert _rel(ex.up_weight.grad, ref["wu"]) < 2e-2
    assert _rel(ex.down_weight.grad, ref["wd"]) < 2e-2


def test_shared_swiglu_native(cuda):
    from saint_llm_b200.models.moe import SwiGLU
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.moe_native import shared_swiglu

    torch.manual_seed(0)
    m = SwiGLU(512, 384, (-10.0, 10.0), 10.0).to(cuda)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(_bf(p * 3))
    h = _bf(torch.randn(333, 512, device=cuda)).requires_grad_(True)
    g = torch.randn(333, 512, device=cuda)
    with backend.eager_mode():
        y0 = m(h)
        y0.backward(g)
    ref = [h.grad.clone()] + [p.grad.clone() for p in m.parameters()]
    h.grad = None
    m.zero_grad()
    y1 = shared_swiglu(h, m)
    y1.float().backward(g)
    assert _rel(y1, y0) < 1e-2
    for got, want in zip([h.grad] + [p.grad for p in m.parameters()], ref, strict=True):
        assert _rel(got, want) < 2e-2


def test_fused_ce(cuda):
    from saint_llm_b200.ops.ce import lm_head_cross_entropy

    torch.manual_seed(0)
    h = torch.randn(2, 300, 256, device=cuda, requires_grad=True)
    w = (torch.randn(1000, 256, device=cuda) * 0.05).requires_grad_(True)
    t = torch.randint(0, 1000, (2, 300), device=cuda)
    for cap in (None, 30.0):
        z = h @ w.t()
        if cap:
            z = cap * torch.tanh(z / cap)
        l0 = F.cross_entropy(z.view(-1, 1000), t.view(-1))
        gh0, gw0 = torch.autograd.grad(l0, (h, w))
        l1 = lm_head_cross_entropy(h, w, t, softcap=cap)
        gh1, gw1 = torch.autograd.grad(l1, (h, w))
        assert abs(l1.item() - l0.item()) < 2e-2
        assert _rel(gh1, gh0) < 3e-2 and _rel(gw1, gw0) < 3e-2


def _tiny_native_vs_eager(cuda, cfg):
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.losses import make_loss_fn

    torch.manual_seed(0)
    model = SaintLLM(cfg).to(cuda)
    x = torch.randint(0, cfg.vocab_size, (2, 64), device=cuda)
    with backend.eager_mode():
        l0 = make_loss_fn(cfg.mtp, moe_cfg=cfg.moe, fused=False)(model, x)
        l0.backward()
    g0 = {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}
    model.zero_grad()
    l1 = make_loss_fn(cfg.mtp, moe_cfg=cfg.moe)(model, x)
    l1.backward()
    torch.cuda.synchronize()
    check_errors(cuda)
    params = dict(model.named_parameters())
    norms = sorted(v.float().norm().item() for v in g0.values())
    floor = 0.4 * norms[len(norms) // 2]  # 0.02 of the median gradient norm, over the 0.05 bound
    rel = {}
    for k, ref in g0.items():
        g = params[k].grad
        assert g is not None and torch.isfinite(g).all(), k
        # error relative to the parameter's own gradient, floored at a fraction of the median
        # gradient norm: some mHC pre-gate gradients cancel to ~1e-7 (the median is ~1e-3),
        # where bf16 rounding alone is larger than the gradient itself
        rel[k] = ((g.float() - ref.float()).norm() / max(ref.float().norm().item(), floor)).item()
    return l0.item(), l1.item(), rel


def test_tiny_model_native_step_per_parameter(cuda):
    """Whole tiny model, native path against the eager fp32 oracle, with every discrete
    choice pinned (hash routing in every MoE layer, CSA top-k covering every block): the
    loss agrees to bf16 precision and EVERY parameter's gradient to a few percent."""
    from saint_llm_b200.config import CSAConfig, ModelConfig

    base = ModelConfig.tiny()
    cfg = base.model_copy(update={
        "moe_use_grouped_gemm": True,
        "moe": base.moe.model_copy(update={"hash_routed_layers": base.n_layers}),
        "csa": CSAConfig(compression_rate=2, indexer_query_heads=2, indexer_head_dim=16, attention_top_k=64),
    })
    l0, l1, rel = _tiny_native_vs_eager(cuda, cfg)
    assert abs(l1 - l0) < 5e-3 * abs(l0), (l0, l1)
    worst = sorted(rel.items(), key=lambda kv: -kv[1])[:5]
    assert worst[0][1] < 0.05, worst


def test_tiny_model_native_step_learned_routing(cuda):
    """Learned routing and indexer selection: bf16 rounding flips a few tokens' expert and
    block choices, which moves many gradients by tens of percent (the test above pins those
    choices and holds every parameter to 5 %).  Here: loss within 1 %, the median parameter
    within 25 % and none completely off."""
    from saint_llm_b200.config import ModelConfig

    cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
    l0, l1, rel = _tiny_native_vs_eager(cuda, cfg)
    assert abs(l1 - l0) < 1e-2 * abs(l0), (l0, l1)
    vals = sorted(rel.values())
    assert vals[len(vals) // 2] < 0.25 and vals[-1] < 1.0, sorted(rel.items(), key=lambda kv: -kv[1])[:5]


def test_smoke_entry(cuda):
    import __graft_entry__

    __graft_entry__.smoke()


def test_gemm_axpby(cuda):
    from saint_llm_b200.ops import gemm

    torch.manual_seed(0)
    a = torch.randn(3, 192, 320, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(3, 256, 320, device=cuda, dtype=torch.bfloat16)
    c = torch.randn(3, 192, 256, device=cuda, dtype=torch.bfloat16)
    out = gemm.gemm_axpby(a, b, c, alpha=0.5, beta=-2.0)
    want = 0.5 * (a.float() @ b.float().transpose(-1, -2)) - 2.0 * c.float()
    assert _rel(out, want) < 1e-2
    out2 = gemm.gemm_axpby(a, c.transpose(-1, -2)[:, :, :320] if False else b, c, alpha=1.0, beta=0.0)
    assert _rel(out2, a.float() @ b.float().transpose(-1, -2)) < 1e-2


@pytest.mark.parametrize("shape", [(3, 256, 512), (2, 512, 256), (4, 1408, 2048), (1, 16, 8192)])
def test_native_newton_schulz(cuda, shape):
    from saint_llm_b200.optim.newton_schulz import hybrid_newton_schulz, native_newton_schulz

    torch.manual_seed(0)
    g = torch.randn(*shape, device=cuda)
    y = (g / (g.norm(dim=(-2, -1), keepdim=True) + 1e-7)).to(torch.bfloat16)
    got = native_newton_schulz(y).float()
    want = torch.stack([hybrid_newton_schulz(m) for m in g])
    # bf16 Newton-Schulz: compare directions of the orthogonalised update
    cos = F.cosine_similarity(got.flatten(1), want.flatten(1), dim=1)
    assert (cos > 0.97).all(), cos


def test_native_muon_step_matches_reference_direction(cuda):
    from saint_llm_b200.optim import Muon

    torch.manual_seed(0)
    w0 = torch.randn(2, 384, 256, device=cuda) * 0.02
    grads = [torch.randn(2, 384, 256, device=cuda) for _ in range(2)]
    a = torch.nn.Parameter(w0.clone())
    b = torch.nn.Parameter(w0.clone().to(torch.bfloat16))
    b.main_grad = torch.zeros(2, 384, 256, device=cuda)
    oa = Muon([a], lr=0.02, ns_impl="reference")
    ob = Muon([b], lr=0.02)
    for g in grads:
        a.grad = g.clone()
        b.main_grad.copy_(g)
        oa.step()
        ob.step()
    da, db = (a.detach() - w0).flatten(1), (b.detach().float() - w0).flatten(1)
    assert (F.cosine_similarity(da, db, dim=1) > 0.97).all()
    assert abs(da.norm().item() / db.norm().item() - 1) < 0.05


def test_shared_expert_group_matches_separate(cuda):
    """Two shared experts fused into one SwiGLU of twice the width == their sum."""
    from saint_llm_b200.models.moe import SwiGLU
    from saint_llm_b200.ops.moe_native import shared_experts, shared_swiglu

    torch.manual_seed(0)
    ex = [SwiGLU(512, 384, (-10.0, 10.0), 10.0).to(cuda) for _ in range(2)]
    with torch.no_grad():
        for e in ex:
            for p in e.parameters():
                p.copy_(_bf(p * 3))
    h = _bf(torch.randn(333, 512, device=cuda)).requires_grad_(True)
    g = torch.randn(333, 512, device=cuda)
    y0 = shared_swiglu(h, ex[0]) + shared_swiglu(h, ex[1])
    y0.float().backward(g)
    ref = [h.grad.clone()] + [p.grad.clone() for e in ex for p in e.parameters()]
    h.grad = None
    for e in ex:
        e.zero_grad()
    y1 = shared_experts(h, ex)
    y1.float().backward(g)
    assert _rel(y1, y0) < 1e-2
    for got, want in zip([h.grad] + [p.grad for e in ex for p in e.parameters()], ref, strict=True):
        assert _rel(got, want) < 2e-2


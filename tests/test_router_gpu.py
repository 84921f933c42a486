"""Fused router forward kernel (+ PyTorch backward) against the eager learned router."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fn", ["sqrt_softplus", "sigmoid"])
@pytest.mark.parametrize("E,k", [(64, 6), (16, 2), (200, 8)])
def test_fused_router_matches_eager(cuda, fn, E, k):
    import torch.nn.functional as F

    from saint_llm_b200.ops.router import fused_route

    torch.manual_seed(0)
    T = 1000
    z = (torch.randn(2, T // 2, E, device=cuda) * 2).requires_grad_(True)
    bias = torch.randn(E, device=cuda) * 0.1
    mbias = torch.randn(2, E, device=cuda) * 0.1
    vis = torch.rand(2, T // 2, device=cuda) < 0.3
    r1, r2 = torch.randn(2, T // 2, k, device=cuda), torch.randn(2, T // 2, E, device=cuda)

    idx, gate, aff = fused_route(z, k, fn, bias, mbias, vis)
    ((gate * r1).sum() + (aff * r2).sum()).backward()
    dz = z.grad.clone()
    z.grad = None

    a = torch.sqrt(F.softplus(z) + 1.0e-12) if fn == "sqrt_softplus" else torch.sigmoid(z)
    biased = a + bias + mbias[vis.long()]
    _, ridx = biased.topk(k, dim=-1)
    g = a.gather(-1, ridx)
    rgate = g / (g.sum(-1, keepdim=True) + 1.0e-12)
    ((rgate * r1).sum() + (a * r2).sum()).backward()
    torch.cuda.synchronize()
    assert torch.equal(idx, ridx)
    assert torch.allclose(aff, a, atol=1e-6, rtol=1e-5)
    assert torch.allclose(gate, rgate, atol=1e-6, rtol=1e-5)
    assert torch.allclose(dz, z.grad, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("with_gate,with_aff", [(True, True), (True, False), (False, True)])
def test_router_backward_kernel_matches_oracle(cuda, mode, with_gate, with_aff):
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.router import route_backward_reference

    torch.manual_seed(mode)
    T, E, k = 300, 64, 6
    z = torch.randn(T, E, device=cuda)
    aff = torch.sqrt(torch.nn.functional.softplus(z) + 1e-12) if mode == 0 else torch.sigmoid(z)
    idx = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(cuda)
    gate = aff.gather(-1, idx)
    gate = gate / (gate.sum(-1, keepdim=True) + 1e-12)
    dg = torch.randn(T, k, device=cuda) if with_gate else None
    da = torch.randn(T, E, device=cuda) if with_aff else None
    dz = torch.empty_like(z)
    backend.ext().router_bwd(z, aff, idx, gate, dg, da, mode, dz)
    want = route_backward_reference(z, aff, idx, gate, dg, da, mode)
    torch.testing.assert_close(dz, want, rtol=1e-5, atol=1e-6)

"""Single-launch AdamW kernel against torch.optim.AdamW (fp32 parameters) and its bf16
parameter path against an fp32 re-computation."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_adamw_multi_matches_torch(cuda):
    from saint_llm_b200.ops.optim_kernels import adamw_step

    torch.manual_seed(0)
    shapes = [(300, 7), (70000,), (1, 1), (129, 1025)]
    ps = [torch.randn(s, device=cuda) for s in shapes]
    ref = [p.clone().requires_grad_(True) for p in ps]
    opt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    states = [{"step": torch.zeros((), device=cuda), "exp_avg": torch.zeros_like(p),
               "exp_avg_sq": torch.zeros_like(p)} for p in ps]
    for step in range(3):
        gs = [torch.randn_like(p) for p in ps]
        for p, g in zip(ps, gs, strict=True):
            p.main_grad = g
        adamw_step(ps, states, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
        for r, g in zip(ref, gs, strict=True):
            r.grad = g.clone()
        opt.step()
    for p, r in zip(ps, ref, strict=True):
        torch.testing.assert_close(p, r.detach(), rtol=1e-5, atol=1e-6)
    assert float(states[0]["step"]) == 3 and states[0]["host_step"] == 3


def test_adamw_multi_bf16_params(cuda):
    from saint_llm_b200.ops.optim_kernels import adamw_step

    torch.manual_seed(1)
    p = torch.randn(4096, device=cuda).to(torch.bfloat16)
    p0 = p.float().clone()
    g = torch.randn(4096, device=cuda)
    p.main_grad = g
    st = [{"step": torch.zeros((), device=cuda), "exp_avg": torch.zeros(4096, device=cuda),
           "exp_avg_sq": torch.zeros(4096, device=cuda)}]
    adamw_step([p], st, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-20, weight_decay=0.1)
    m = 0.1 * g
    v = 0.05 * g * g
    want = p0 * (1 - 1e-4) - 1e-3 * (m / 0.1) / ((v / 0.05).sqrt() + 1e-20)
    # one bf16 rounding step apart at most (scalar constants round differently in fp32)
    torch.testing.assert_close(p.float(), want.to(torch.bfloat16).float(), rtol=8e-3, atol=1e-6)

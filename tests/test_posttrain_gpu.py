"""Fused per-token log-probabilities (LM-head GEMM + CE kernels) against fp32 PyTorch."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cap", [None, 30.0])
def test_token_logprobs_values_and_grads(cuda, cap):
    from saint_llm_b200.ops.ce import token_logprobs

    torch.manual_seed(0)
    h = torch.randn(3, 70, 256, device=cuda, requires_grad=True)
    w = (torch.randn(1000, 256, device=cuda) * 0.05).requires_grad_(True)
    t = torch.randint(0, 1000, (3, 70), device=cuda)
    g = torch.randn(3, 70, device=cuda)
    z = h.bfloat16().float() @ w.bfloat16().float().t()
    if cap:
        z = cap * torch.tanh(z / cap)
    ref = F.log_softmax(z, -1).gather(-1, t[..., None]).squeeze(-1)
    gh0, gw0 = torch.autograd.grad((ref * g).sum(), (h, w))
    got = token_logprobs(h, w, t, softcap=cap)
    gh1, gw1 = torch.autograd.grad((got * g).sum(), (h, w))
    assert (got - ref).abs().max() < 2e-2
    for a, b in ((gh1, gh0), (gw1, gw0)):
        assert (a.float() - b).norm() / b.norm() < 3e-2


def test_policy_logprobs_native_model(cuda):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.ops import backend
    from saint_llm_b200.posttrain import gather_token_logprobs, policy_token_logprobs

    torch.manual_seed(0)
    model = SaintLLM(ModelConfig.tiny()).to(cuda)
    tokens = torch.randint(0, 512, (2, 64), device=cuda)
    lp = policy_token_logprobs(model, tokens)
    with backend.eager_mode():
        ref = gather_token_logprobs(model(tokens)["logits"], tokens)
    assert lp.shape == ref.shape and (lp - ref).abs().max() < 0.1

"""``saint_llm_b200.kernels`` on the B200: the native indexer, mHC carry and block-scaled FP8
GEMM behind the reference package's names, against their fp32 definitions."""

import pytest
import torch

from saint_llm_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-12)).item()


@pytest.mark.parametrize("vis", [False, True])
def test_native_indexer_scores_and_topk(cuda, vis):
    from saint_llm_b200.ops.gemm import check_errors

    torch.manual_seed(0)
    b, t, h, c, nb, m = 2, 200, 4, 64, 50, 4
    q = torch.randn(b, t, h, c, device=cuda)
    k = torch.randn(b, nb, c, device=cuda)
    w = torch.rand(b, t, h, device=cuda)
    vb = torch.rand(b, nb, device=cuda) if vis else None
    qr, kr = q.to(torch.bfloat16).float(), k.to(torch.bfloat16).float()  # the kernel's operand rounding
    got = K.lightning_indexer_scores(q, k, w, vb)
    torch.cuda.synchronize()
    check_errors(cuda)
    want = K.lightning_indexer_scores_reference(qr, kr, w, vb)
    assert torch.isfinite(got).all() and _rel(got, want) < 1e-3
    ids = K.lightning_indexer_topk(q, k, w, 8, m, vb)
    want_ids = K.lightning_indexer_topk_reference(qr, kr, w, 8, m, vb)
    torch.cuda.synchronize()
    check_errors(cuda)
    assert ids.shape == want_ids.shape and torch.equal(ids < 0, want_ids < 0)
    # the same picks up to ties: compare the scores of the picked blocks
    masked = want.masked_fill(~K._block_visible(t, nb, m, cuda), float("-inf"))
    pick = lambda i: masked.gather(-1, i.clamp(min=0)).masked_fill(i < 0, 0.0)  # noqa: E731
    assert (pick(ids) - pick(want_ids)).abs().max().item() <= 1e-3 * masked[torch.isfinite(masked)].abs().max().item()


def test_native_mhc_carry(cuda):
    torch.manual_seed(1)
    b, t, n, d = 2, 70, 4, 256
    x = torch.randn(b, t, n, d, device=cuda).to(torch.bfloat16).requires_grad_(True)
    o = torch.randn(b, t, d, device=cuda).to(torch.bfloat16).requires_grad_(True)
    b_l = torch.randn(b, t, n, n, device=cuda).requires_grad_(True)
    c_l = torch.randn(b, t, n, device=cuda).requires_grad_(True)
    y = K.mhc_carry(b_l, c_l, x, o)
    assert y.dtype == torch.bfloat16
    leaves = [b_l, c_l, x, o]
    ref_leaves = [p.detach().float().requires_grad_(True) for p in leaves]
    ref = K.mhc_carry_reference(*ref_leaves)
    assert _rel(y, ref) < 1e-2
    g = torch.randn(ref.shape, device=cuda)
    y.float().backward(g)
    ref.backward(g)
    for a, r in zip(leaves, ref_leaves, strict=True):
        assert _rel(a.grad, r.grad) < 2e-2


def test_native_fp8_gemm(cuda):
    from saint_llm_b200.ops import backend

    assert K.is_fp8_gemm_supported(cuda)
    torch.manual_seed(4)
    x = (torch.randn(2, 200, 512, device=cuda) * 0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(384, 512, device=cuda) * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = K.fp8_gemm(x, w)
    with backend.eager_mode():
        emu = K.fp8_gemm(x.detach(), w.detach())  # the same quantisation as a dequantised matmul
    assert y.dtype == torch.bfloat16 and _rel(y, emu) < 1e-2
    g = torch.randn_like(y)
    y.backward(g)
    assert _rel(x.grad, (g.float().reshape(-1, 384) @ w.detach().float()).reshape(x.shape)) < 1e-2
    assert _rel(w.grad, g.float().reshape(-1, 384).t() @ x.detach().float().reshape(-1, 512)) < 1e-2

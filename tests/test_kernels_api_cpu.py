"""The kernel-level public functions (``saint_llm_b200.kernels``) on CPU: their fp32
definitions against the reference package's eager functions, the block-causal top-k rules,
and the FP8 GEMM's quantised forward and straight-through backward."""

import pytest
import torch

from saint_llm_b200 import kernels as K


def _indexer_inputs(seed=0, b=2, t=24, h=3, c=16, nb=6):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(b, t, h, c, generator=g), torch.randn(b, nb, c, generator=g),
            torch.rand(b, t, h, generator=g), torch.rand(b, nb, generator=g))


def test_definitions_match_the_reference_package(ref_pkgs):
    from saint_llm_kernels import attention as ra
    from saint_llm_kernels import mhc as rm

    q, k, w, vis = _indexer_inputs()
    for v in (None, vis):
        torch.testing.assert_close(K.lightning_indexer_scores_reference(q, k, w, v),
                                   ra.lightning_indexer_scores_reference(q, k, w, v))
        assert torch.equal(K.lightning_indexer_topk_reference(q, k, w, 3, 4, v),
                           ra.lightning_indexer_topk_reference(q, k, w, 3, 4, v))
    g = torch.Generator().manual_seed(1)
    b_l, c_l = torch.randn(2, 5, 4, 4, generator=g), torch.randn(2, 5, 4, generator=g)
    x, o = torch.randn(2, 5, 4, 8, generator=g), torch.randn(2, 5, 8, generator=g)
    torch.testing.assert_close(K.mhc_carry_reference(b_l, c_l, x, o), rm.mhc_carry_reference(b_l, c_l, x, o))


def test_indexer_topk_block_causal_rules():
    q, k, w, _ = _indexer_inputs(t=12, nb=3)
    ids = K.lightning_indexer_topk(q, k, w, top_k=2, block_size_m=4)
    assert ids.shape == (2, 12, 2)
    # block s (tokens 4s .. 4s+3) becomes visible at query 4s+4: none before t=4, one until t=8
    assert (ids[:, :4] == -1).all()
    assert (ids[:, 4:8, 0] == 0).all() and (ids[:, 4:8, 1] == -1).all()
    assert ((ids[:, 8:] >= 0) & (ids[:, 8:] <= 1)).all()
    s = K.lightning_indexer_scores(q, k, w)
    best = s[:, 8:, :2].argmax(-1)
    assert torch.equal(ids[:, 8:, 0], best)
    assert K.lightning_indexer_topk(q, k, w, top_k=0, block_size_m=4).shape == (2, 12, 0)
    assert K.lightning_indexer_topk(q, k[:, :0], w, top_k=2, block_size_m=4).shape == (2, 12, 0)
    # more requested than exist: k_eff = n_blocks
    assert K.lightning_indexer_topk(q, k, w, top_k=9, block_size_m=4).shape == (2, 12, 3)


def test_mhc_carry_cpu_is_differentiable():
    g = torch.Generator().manual_seed(2)
    b_l = torch.randn(1, 3, 2, 2, generator=g, requires_grad=True)
    c_l = torch.randn(1, 3, 2, generator=g, requires_grad=True)
    x = torch.randn(1, 3, 2, 4, generator=g, requires_grad=True)
    o = torch.randn(1, 3, 4, generator=g, requires_grad=True)
    y = K.mhc_carry(b_l, c_l, x, o)
    torch.testing.assert_close(y[0, 1, 0], b_l[0, 1, 0, 0] * x[0, 1, 0] + b_l[0, 1, 0, 1] * x[0, 1, 1]
                               + c_l[0, 1, 0] * o[0, 1])
    y.sum().backward()
    torch.testing.assert_close(o.grad, c_l.detach().sum(-1, keepdim=True).expand_as(o))


def test_fp8_gemm_quantised_forward_and_ste_backward():
    from saint_llm_b200.ops import fp8

    assert not K.is_fp8_gemm_supported(torch.device("cpu"))
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(3, 5, 256, generator=g) * 0.5).requires_grad_(True)
    w = (torch.randn(128, 256, generator=g) * 0.05).requires_grad_(True)
    y = K.fp8_gemm(x, w, out_dtype=torch.float32)
    assert y.shape == (3, 5, 128) and y.dtype == torch.float32
    want = fp8.quantize_rows(x.detach().reshape(-1, 256)).dequantize() @ fp8.quantize_blocks(w.detach()).dequantize().t()
    torch.testing.assert_close(y.reshape(-1, 128), want.to(torch.bfloat16).float())
    exact = x.detach().reshape(-1, 256) @ w.detach().t()
    assert (y.detach().reshape(-1, 128) - exact).norm() < 0.08 * exact.norm()
    gy = torch.randn(y.shape, generator=g)
    y.backward(gy)
    torch.testing.assert_close(x.grad, (gy.reshape(-1, 128) @ w.detach()).reshape(x.shape))
    torch.testing.assert_close(w.grad, gy.reshape(-1, 128).t() @ x.detach().reshape(-1, 256))
    with pytest.raises(ValueError, match="E4M3"):
        K.fp8_gemm(x, w, weight_fmt=K.Fp8Format.E5M2)
    with pytest.raises(ValueError, match="divisible by 128"):
        K.fp8_gemm(torch.randn(2, 100), torch.randn(128, 100))
    with pytest.raises(ValueError, match="K mismatch"):
        K.fp8_gemm(torch.randn(2, 128), torch.randn(128, 256))


def test_public_names_cover_the_reference_kernels_package(ref_pkgs):
    import saint_llm_kernels

    assert set(saint_llm_kernels.__all__) <= set(K.__all__)
    for name in K.__all__:
        assert hasattr(K, name)

"""Native tcgen05 GEMM vs a plain fp32 PyTorch reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().transpose(-1, -2)


def _close(x, y, tol=2e-2):
    err = (x.float() - y.float()).abs().max().item()
    scale = y.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (300, 200, 192), (4096, 2048, 2048),
                                   (1, 17, 64), (1000, 1408, 2048)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_layouts(cuda, m, n, k, a_t, b_t):
    from saint_llm_b200.ops import gemm

    torch.manual_seed(0)
    a = torch.randn(k, m, device=cuda, dtype=torch.bfloat16).t() if a_t else torch.randn(m, k, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(k, n, device=cuda, dtype=torch.bfloat16).t() if b_t else torch.randn(n, k, device=cuda, dtype=torch.bfloat16)
    out = gemm.gemm_nt(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    _close(out, _ref(a, b), 1e-3)
    out16 = gemm.gemm_nt(a, b)
    _close(out16, _ref(a, b))


def test_gemm_accumulate_and_batched(cuda):
    from saint_llm_b200.ops import gemm

    torch.manual_seed(1)
    a = torch.randn(5, 192, 320, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(5, 130, 320, device=cuda, dtype=torch.bfloat16)
    acc = torch.randn(5, 192, 130, device=cuda, dtype=torch.float32)
    want = acc + _ref(a, b)
    gemm.gemm_nt(a, b, out=acc, accumulate=True)
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    _close(acc, want, 1e-3)
    # batched a @ b with b row-major (MN-major operand)
    x = torch.randn(7, 128, 256, device=cuda, dtype=torch.bfloat16)
    y = torch.randn(7, 256, 384, device=cuda, dtype=torch.bfloat16)
    _close(gemm.bmm(x, y), x.float() @ y.float(), 1e-3)


@pytest.mark.parametrize("accumulate", [False, True])
@pytest.mark.parametrize("m,n,k", [(1024, 256, 4096), (24, 8192, 4096), (4096, 24, 8192), (200, 100, 2048)])
def test_gemm_split_k_skinny(cuda, m, n, k, accumulate):
    """Few output tiles and long K: the K-split path (TMA reduce-add into fp32)."""
    from saint_llm_b200.ops import gemm

    torch.manual_seed(2)
    # weight-gradient layout: both operands MN-major (token dimension is K)
    a = torch.randn(k, m, device=cuda, dtype=torch.bfloat16).t()
    b = torch.randn(k, n, device=cuda, dtype=torch.bfloat16).t()
    base = torch.randn(m, n, device=cuda, dtype=torch.float32)
    out = base.clone()
    gemm.gemm_nt(a, b, out=out, accumulate=accumulate)
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    want = _ref(a, b) + (base if accumulate else 0)
    _close(out, want, 1e-3)


@pytest.mark.parametrize("out_dtype,accumulate", [(torch.bfloat16, False), (torch.float32, False),
                                                   (torch.float32, True)])
@pytest.mark.parametrize("m,n,k", [(24, 8192, 4096), (64, 2048, 1024), (256, 512, 512)])
@pytest.mark.parametrize("batch1", [False, True])
def test_gemm_skinny_k_major_fixed_order(cuda, m, n, k, out_dtype, accumulate, batch1):
    """Skinny K-major products (decode projections): K slices into separate fp32 partials
    summed in a fixed order.  Checked against fp32, bit-identical across two calls, and
    the same when the operands arrive as (1, rows, K) batch-1 views."""
    from saint_llm_b200.ops import gemm

    torch.manual_seed(4)
    a = torch.randn(m, k, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=cuda, dtype=torch.bfloat16)
    base = torch.randn(m, n, device=cuda, dtype=torch.float32)
    want = _ref(a, b) + (base if accumulate else 0)
    if batch1:
        a, b = a.unsqueeze(0), b.unsqueeze(0)

    def run():
        shape = (1, m, n) if batch1 else (m, n)
        if accumulate:
            out = base.clone().reshape(shape)
            gemm.gemm_nt(a, b, out=out, accumulate=True)
        else:
            out = gemm.gemm_nt(a, b, out_dtype=out_dtype)
        torch.cuda.synchronize()
        gemm.check_errors(cuda)
        return out.reshape(m, n)

    o1, o2 = run(), run()
    _close(o1, want, 1e-3 if out_dtype == torch.float32 else 2e-2)
    assert torch.equal(o1, o2), "split-K partial sum is not deterministic"


def test_gemm_bf16_output_view_with_row_stride(cuda):
    """bf16 output written through a TMA map into a column slice of a wider buffer."""
    from saint_llm_b200.ops import gemm

    torch.manual_seed(3)
    a = torch.randn(300, 256, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(200, 256, device=cuda, dtype=torch.bfloat16)
    wide = torch.zeros(300, 520, device=cuda, dtype=torch.bfloat16)
    gemm.gemm_nt(a, b, out=wide[:, 8:208])
    torch.cuda.synchronize()
    _close(wide[:, 8:208], _ref(a, b))
    assert wide[:, :8].abs().sum() == 0 and wide[:, 208:].abs().sum() == 0


@pytest.mark.parametrize("batch,r,k", [(3, 1408, 2048), (2, 200, 256), (1, 520, 64)])
def test_symmetric_gemm_and_axpby(cuda, batch, r, k):
    """Symmetric outputs computed on the upper tiles only; the skipped tiles are filled from the
    epilogue with the transposed values, so the result is exactly symmetric and its upper
    triangle equals the full product's."""
    from saint_llm_b200.ops.gemm import gemm_axpby, gemm_nt

    torch.manual_seed(0)
    y = (torch.randn(batch, r, k, device=cuda) / k ** 0.5).to(torch.bfloat16)
    g = gemm_nt(y, y, symmetric=True)
    ref = y.float() @ y.float().transpose(-1, -2)
    assert torch.equal(g, g.transpose(-1, -2))
    assert ((g.float() - ref).norm() / ref.norm()).item() < 1e-2
    p = gemm_axpby(g, g, g, alpha=-1.5, beta=0.5, symmetric=True)
    pref = -1.5 * g.float() @ g.float() + 0.5 * g.float()
    assert torch.equal(p, p.transpose(-1, -2))
    assert ((p.float() - pref).norm() / pref.norm()).item() < 1e-2
    full = gemm_nt(y, y)
    up = torch.triu(torch.ones(r, r, dtype=torch.bool, device=cuda))
    assert torch.equal(g[:, up], full[:, up])

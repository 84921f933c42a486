"""Block-scaled FP8: native quantisation kernels vs the PyTorch oracle (identical bytes and
scales) and the tcgen05 block-scaled GEMM vs a plain fp32 product of the dequantised
operands."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _operand(rows, k, device, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    # row and column-block magnitudes spread over many binades exercise every scale
    x = x * torch.exp2(torch.randint(-12, 12, (rows, 1), generator=g).float())
    x = x * torch.exp2(torch.randint(-4, 4, (1, k // 128), generator=g).float()).repeat_interleave(128, 1)
    return x.to(torch.bfloat16).to(device)


def _sf_byte(sf, r, kb, kblocks):
    """Scale byte of row r, K block kb: 512-byte chunks per (128 rows, 4 K blocks)."""
    groups = (kblocks + 3) // 4
    return int(sf[(r // 128 * groups + kb // 4) * 512 + 16 * (r % 32) + 4 * ((r % 128) // 32) + kb % 4])


@pytest.mark.parametrize("m,k", [(300, 512), (128, 128), (1, 256), (4096, 2048), (200, 640)])
def test_quant_rows_matches_oracle(cuda, m, k):
    from saint_llm_b200.ops import fp8

    x = _operand(m, k, cuda, 0)
    nat = fp8.quantize_rows(x)
    ref = fp8._oracle_rows(x.cpu())
    torch.cuda.synchronize()
    assert torch.equal(nat.scale.cpu(), ref.scale)
    assert torch.equal(nat.q.cpu(), ref.q)
    sf = nat.sf.cpu()
    kb_n = k // 128
    for r in {0, m // 2, m - 1}:
        for kb in {0, kb_n - 1}:
            e = int(torch.log2(ref.scale[r, kb]).item())
            assert _sf_byte(sf, r, kb, kb_n) == e + 127


@pytest.mark.parametrize("n,k", [(128, 128), (384, 512), (2048, 2048)])
def test_quant_blocks_matches_oracle(cuda, n, k):
    from saint_llm_b200.ops import fp8

    w = _operand(n, k, cuda, 1)
    nat = fp8.quantize_blocks(w)
    ref = fp8._oracle_blocks(w.cpu())
    torch.cuda.synchronize()
    assert torch.equal(nat.scale.cpu(), ref.scale)
    assert torch.equal(nat.q.cpu(), ref.q)
    sf = nat.sf.cpu()
    kb_n = k // 128
    e = int(torch.log2(ref.scale[-1, -1]).item())
    assert _sf_byte(sf, n - 1, kb_n - 1, kb_n) == e + 127


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (300, 384, 512), (1, 256, 256), (4096, 2048, 2048),
                                   (1000, 1408, 2048), (256, 256, 1408), (130, 128, 640)])
def test_gemm_fp8_matches_fp32(cuda, m, n, k):
    from saint_llm_b200.ops import fp8, gemm

    a = fp8.quantize_rows(_operand(m, k, cuda, 2))
    b = fp8.quantize_blocks(_operand(n, k, cuda, 3))
    out = fp8.gemm(a, b)
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    ref = a.dequantize() @ b.dequantize().t()
    err = (out.float() - ref).abs()
    # bf16 output rounding: relative to each row's magnitude
    row_scale = ref.abs().amax(1, keepdim=True) + 1e-30
    assert (err / row_scale).max().item() < 1e-2
    assert torch.isfinite(out).all()


def test_fp8_linear_forward_and_ste_backward(cuda):
    from saint_llm_b200.ops import fp8
    from saint_llm_b200.ops.linear import fp8_linear, linear

    torch.manual_seed(4)
    x = (torch.randn(2, 200, 512, device=cuda) * 0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(384, 512, device=cuda) * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = fp8_linear(x, w)
    ref = fp8.quantize_rows(x.detach().reshape(-1, 512)).dequantize() @ fp8.quantize_blocks(w.detach()).dequantize().t()
    assert (y.float().reshape(-1, 384) - ref).abs().max().item() < 1e-2 * ref.abs().max().item()
    # quantisation error of the whole recipe against the exact bf16 product stays small
    exact = x.detach().float().reshape(-1, 512) @ w.detach().float().t()
    assert (y.float().reshape(-1, 384) - exact).norm().item() < 0.08 * exact.norm().item()
    g = torch.randn_like(y)
    y.backward(g)
    x2 = x.detach().clone().requires_grad_(True)
    w2 = w.detach().clone().requires_grad_(True)
    linear(x2, w2).backward(g)
    assert torch.allclose(x.grad.float(), x2.grad.float(), atol=1e-2, rtol=1e-2)
    assert torch.allclose(w.grad.float(), w2.grad.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("used", [8, 3])
def test_fp8_routed_experts_match_bf16(cuda, used):
    """Grouped FP8 GEMMs (SwiGLU epilogue, then the down projection) against the bf16 grouped
    path; ``used`` < E leaves experts without rows (no tiles)."""
    from saint_llm_b200.ops import gemm, moe_native
    from saint_llm_b200.ops.moe import GroupedSwiGLUExperts

    torch.manual_seed(5)
    E, D, I, T, k = 8, 256, 384, 300, 2
    ex = GroupedSwiGLUExperts(D, I, E).to(cuda).to(torch.bfloat16)
    h = torch.randn(T, D, device=cuda, dtype=torch.bfloat16)
    idx = torch.stack([torch.randperm(used)[:k] for _ in range(T)]).to(cuda)
    gate = torch.rand(T, k, device=cuda)
    with torch.no_grad():
        ref = moe_native.routed_experts(h, idx, gate, ex)
        got = moe_native.routed_experts_fp8(h, idx, gate, moe_native.Fp8ExpertWeights(ex))
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    assert torch.isfinite(got).all()
    rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 0.08, rel


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fake_quant_fp4_kernel_matches_oracle(cuda, dtype):
    """Native MX FP4 straight-through quantiser against the PyTorch statement on the same
    device (same scale rule, E2M1 rounding with ties to the smaller magnitude)."""
    from saint_llm_b200.ops.linear import fake_quant_fp4
    from saint_llm_b200.ops.quant import fake_quant_fp4_mx

    torch.manual_seed(9)
    x = (torch.randn(64, 256, device=cuda) * torch.exp2(torch.randint(-8, 8, (64, 1), device=cuda).float()))
    x[0, :32] = 0.0                                   # an all-zero block
    x[1, :32] = torch.linspace(-6, 6, 32, device=cuda)  # exact E2M1 levels and ties
    x = x.to(dtype).requires_grad_(True)
    got = fake_quant_fp4(x, 32)
    want = fake_quant_fp4_mx(x.detach(), block_size=32, axis=-1)
    torch.cuda.synchronize()
    mismatch = (got.detach() != want).float().mean().item()
    assert mismatch < 1e-3, mismatch  # at most a rare log2 rounding edge
    g = torch.randn_like(got)
    got.backward(g)
    assert torch.equal(x.grad, g)  # straight-through

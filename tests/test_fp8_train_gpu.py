"""Block-scaled FP8 training path: the fused gather + quantisation and gate/up interleave
kernels against the plain quantisation kernels (identical bytes), the weight cache's
refresh rule, the FP8 forward of routed and shared experts against an fp32 product of the
dequantised operands, and a whole FP8 training step against the bf16 step."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_gather_quant_rows_equals_quant_of_gathered(cuda):
    from saint_llm_b200.ops import fp8, gemm

    torch.manual_seed(0)
    T, D, M = 50, 512, 300
    h = (torch.randn(T, D, device=cuda) * torch.exp2(torch.randint(-6, 6, (T, 1), device=cuda).float())).to(
        torch.bfloat16)
    row_token = torch.randint(-1, T, (M,), device=cuda, dtype=torch.int32)
    got = fp8.gather_quantize_rows(h, row_token, M)
    rows = torch.where(row_token[:, None] >= 0, h[row_token.clamp(min=0).long()], torch.zeros_like(h[:1]))
    want = fp8.quantize_rows(rows.contiguous())
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    assert torch.equal(got.q, want.q)
    assert torch.equal(got.sf, want.sf)


def test_quant_blocks_gu_equals_interleaved_quant(cuda):
    from saint_llm_b200.ops import fp8

    torch.manual_seed(1)
    E, I, D = 3, 192, 256
    wg = torch.randn(E, I, D, device=cuda).to(torch.bfloat16)
    wu = (torch.randn(E, I, D, device=cuda) * 3).to(torch.bfloat16)
    inter = torch.stack([wg.reshape(E, I // 64, 64, D), wu.reshape(E, I // 64, 64, D)], 2).reshape(E * 2 * I, D)
    want = fp8.quantize_blocks(inter.contiguous())
    got = fp8.Fp8WeightCache([wg, wu], "gu").get()
    torch.cuda.synchronize()
    assert torch.equal(got.q, want.q)
    # scale bytes: compare the slots that hold a scale (a 512-byte chunk has four K-block
    # slots per row; with K = 256 two of them are unused padding)
    n, kb_n = E * 2 * I, D // 128
    groups = (kb_n + 3) // 4
    used = torch.tensor([(r // 128 * groups + kb // 4) * 512 + 16 * (r % 32) + 4 * ((r % 128) // 32) + kb % 4
                         for r in range(n) for kb in range(kb_n)], device=cuda)
    assert torch.equal(got.sf[used], want.sf[used])


def test_weight_cache_refreshes_on_epoch_and_version(cuda):
    from saint_llm_b200.ops import fp8

    w = torch.randn(256, 256, device=cuda).to(torch.bfloat16)
    cache = fp8.Fp8WeightCache([w], "rows")
    q0 = cache.get().q.clone()
    with torch.no_grad():
        w.data.mul_(2.0)  # .data: no version bump -- only the epoch tells the cache
    assert torch.equal(cache.get().q, q0)
    fp8.bump_weight_epoch()
    q1 = cache.get().q.clone()
    assert torch.equal(q1, fp8.quantize_blocks(w).q)
    w.add_(1.0)  # a version bump alone also refreshes
    assert torch.equal(cache.get().q, fp8.quantize_blocks(w).q)


def _dq(op):
    return op.dequantize().float()


def test_routed_experts_fp8_training_forward_and_backward(cuda):
    """Training-mode FP8 forward of a routed pool equals the fp32 product of the dequantised
    operands; its backward is the bf16 straight-through backward (close to the bf16 path)."""
    from saint_llm_b200.ops import fp8, gemm, moe_native
    from saint_llm_b200.ops.moe import GroupedSwiGLUExperts

    torch.manual_seed(2)
    E, D, I, T, k = 8, 256, 384, 320, 2
    ex = GroupedSwiGLUExperts(D, I, E).to(cuda).to(torch.bfloat16)
    ex.linear_quant = "fp8"
    ex.fp8_weight_cache = "always"
    ref_ex = GroupedSwiGLUExperts(D, I, E).to(cuda).to(torch.bfloat16)
    ref_ex.load_state_dict(ex.state_dict())
    h = torch.randn(T, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    idx = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(cuda)
    gate = torch.rand(T, k, device=cuda, requires_grad=True)
    out = moe_native.routed_experts(h, idx, gate, ex)
    # oracle: dequantised FP8 operands in fp32
    wq = fp8.quantize_blocks
    y_ref = torch.zeros(T, D, device=cuda)
    hq = _dq(fp8.quantize_rows(h.detach()))
    for e in range(E):
        g_ = hq @ _dq(wq(ex.gate_weight[e].detach())).t()
        u_ = hq @ _dq(wq(ex.up_weight[e].detach())).t()
        a = torch.nn.functional.silu(g_.clamp(max=ex.clamp_gate_max)) * u_.clamp(*ex.clamp_linear)
        a = _dq(fp8.quantize_rows(a.to(torch.bfloat16)))
        ye = a @ _dq(wq(ex.down_weight[e].detach())).t()
        w_e = (gate.detach() * (idx == e)).sum(1, keepdim=True)
        y_ref += w_e * ye
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    rel = ((out.float() - y_ref).norm() / y_ref.norm()).item()
    assert rel < 2e-2, rel
    g = torch.randn_like(out)
    out.backward(g)
    h2 = h.detach().clone().requires_grad_(True)
    gate2 = gate.detach().clone().requires_grad_(True)
    moe_native.routed_experts(h2, idx, gate2, ref_ex).backward(g)
    for a, b in ((h.grad, h2.grad), (ex.down_weight.grad, ref_ex.down_weight.grad),
                 (ex.gate_weight.grad, ref_ex.gate_weight.grad)):
        r = ((a.float() - b.float()).norm() / b.float().norm()).item()
        assert r < 0.1, r  # the saved pre-activations come from the FP8 forward


def test_shared_experts_fp8_forward(cuda):
    from saint_llm_b200.models.linear import Fp8Linear
    from saint_llm_b200.models.moe import SwiGLU
    from saint_llm_b200.ops import fp8, moe_native

    torch.manual_seed(3)
    D, I, T = 256, 256, 384

    def factory(i, o, *, bias=True):
        return Fp8Linear(i, o, bias=bias, use_real_fp8_gemm=True)

    ex = [SwiGLU(D, I, (-10.0, 10.0), 10.0, linear_factory=factory).to(cuda).to(torch.bfloat16) for _ in range(2)]
    h = (torch.randn(T, D, device=cuda) * 0.5).to(torch.bfloat16)
    out = moe_native.shared_experts(h, ex)
    assert getattr(ex[0], "_fp8_shared_gu", None) is not None  # the FP8 path ran
    hq = _dq(fp8.quantize_rows(h))
    want = torch.zeros(T, D, device=cuda)
    acts = []
    for e in ex:
        g_ = hq @ _dq(fp8.quantize_blocks(e.gate_proj.weight.detach())).t()
        u_ = hq @ _dq(fp8.quantize_blocks(e.up_proj.weight.detach())).t()
        acts.append(torch.nn.functional.silu(g_.clamp(max=10.0)) * u_.clamp(-10.0, 10.0))
    a = _dq(fp8.quantize_rows(torch.cat(acts, 1).to(torch.bfloat16)))
    wd = torch.cat([e.down_proj.weight.detach() for e in ex], 1)
    want = a @ _dq(fp8.quantize_blocks(wd)).t()
    rel = ((out.float() - want).norm() / want.norm()).item()
    assert rel < 2e-2, rel


def test_fp8_training_step_tracks_bf16(cuda):
    """Three optimizer steps of the 2-layer config-3 model in FP8 and in bf16 from the same
    initialisation and data: the FP8 losses follow the bf16 losses."""
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.launch import build_training

    torch.manual_seed(6)
    data = [torch.randint(0, 32768, (2, 1, 512), device=cuda) for _ in range(3)]
    losses = {}
    for quant in ("bf16", "fp8"):
        cfg = ModelConfig.bench_16b().model_copy(update={"n_layers": 2, "linear_quant": quant})
        job = build_training(cfg, RunConfig(grad_accum=2, micro_batch=1, seq_len=512, seed=0), cuda)
        losses[quant] = [float(job.step.run_device(d).item()) for d in data]
        torch.cuda.synchronize()
        check_errors(cuda)
        del job
        torch.cuda.empty_cache()
    for a, b in zip(losses["bf16"], losses["fp8"], strict=True):
        assert abs(a - b) < 0.03 * a, losses

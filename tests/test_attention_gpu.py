"""Fused tcgen05 attention (window + sink + softcap, HCA / CSA compressed branch) against a
plain fp32 PyTorch reference of the same math, forward and backward."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, kv, sink, sel, mode, m, window, softcap):
    b, t, h, d = q.shape
    q, k, v = q.float(), k.float(), v.float()
    s = torch.einsum("bthd,bsd->bhts", q, k) / math.sqrt(d)
    qpos = torch.arange(t, device=q.device).view(-1, 1)
    kpos = torch.arange(t, device=q.device).view(1, -1)
    vis = (kpos <= qpos) & (qpos - kpos < window)
    amax = s.detach().abs().masked_fill(~vis, 0).amax()
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    s = s.masked_fill(~vis, float("-inf"))
    if sink is not None:
        s = torch.cat([s, sink.float().view(1, h, 1, 1).expand(b, h, t, 1)], -1)
    p = torch.softmax(s, -1)
    if sink is not None:
        p = p[..., :-1]
    o = torch.einsum("bhts,bsd->bthd", p, v)
    if mode:
        kvf = kv.float()
        n = kvf.shape[1]
        sc = torch.einsum("bthd,bnd->bhtn", q, kvf) / math.sqrt(d)
        if mode == 1:
            visc = ((torch.arange(n, device=q.device) * m + m - 1).view(1, -1) < qpos).view(1, 1, t, n)
        else:
            visc = sel.view(b, 1, t, n)
        sc = sc.masked_fill(~visc, float("-inf"))
        if mode == 1 and sink is not None:
            sc = torch.cat([sc, sink.float().view(1, h, 1, 1).expand(b, h, t, 1)], -1)
            pc = torch.softmax(sc, -1)[..., :-1]
        else:
            pc = torch.nan_to_num(torch.softmax(sc, -1), nan=0.0)
        o = o + torch.einsum("bhtn,bnd->bthd", pc, kvf)
    return o, amax


def _close(x, y, tol):
    err = (x.float() - y.float()).abs().max().item()
    scale = y.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


CASES = [
    # (B, T, H, d, window, mode, m, sink, softcap)
    (1, 256, 2, 128, 128, 0, 1, True, None),
    (2, 300, 3, 128, 64, 0, 1, False, 30.0),
    (1, 384, 2, 64, 200, 1, 8, True, None),
    (2, 260, 2, 128, 128, 2, 4, False, None),
    (1, 200, 2, 32, 16, 1, 16, True, 20.0),
]


@pytest.mark.parametrize("case", CASES)
def test_fused_attention_matches_reference(cuda, case):
    from saint_llm_b200.ops import gemm
    from saint_llm_b200.ops.attention import fused_attention

    b, t, h, d, window, mode, m, with_sink, softcap = case
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda *s: (torch.randn(*s, device=cuda, generator=g) * 1.5).to(torch.bfloat16)  # noqa: E731
    q, k, v = mk(b, t, h, d), mk(b, t, d), mk(b, t, d)
    n = t // m if mode else 0
    kv = mk(b, n, d) if mode else None
    sink = (torch.randn(h, device=cuda, generator=g)).to(torch.bfloat16) if with_sink else None
    sel_bool, sel = None, None
    if mode == 2:
        qpos = torch.arange(t, device=cuda).view(-1, 1)
        causal = (torch.arange(n, device=cuda) * m + m - 1).view(1, -1) < qpos
        sel_bool = (torch.rand(b, t, n, device=cuda, generator=g) < 0.5) & causal
        top = torch.where(sel_bool, torch.arange(n, device=cuda).expand(b, t, n), torch.full_like(sel_bool, -1,
                                                                                                dtype=torch.long))
        sel = torch.empty(b, t, (n + 31) // 32, dtype=torch.int32, device=cuda)
        from saint_llm_b200.ops import backend

        backend.ext().csa_select_mask(top.contiguous(), n, sel, gemm.error_word(cuda))
    leaves = [x.detach().clone().requires_grad_(True) if x is not None else None for x in (q, k, v, kv, sink)]
    ml = torch.zeros((), device=cuda)
    out = fused_attention(leaves[0], leaves[1], leaves[2], window=window, sink=leaves[4], softcap=softcap,
                          kv=leaves[3], mode=mode, m=m, sel=sel, maxlogit=ml)
    ref_leaves = [x.detach().clone().float().requires_grad_(True) if x is not None else None
                  for x in (q, k, v, kv, sink)]
    ref, amax = _ref(ref_leaves[0], ref_leaves[1], ref_leaves[2], ref_leaves[3], ref_leaves[4], sel_bool, mode, m,
                     window, softcap)
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    _close(out, ref, 2e-2)
    assert abs(float(ml) - float(amax)) <= 1e-2 * float(amax) + 1e-3
    dout = torch.randn(out.shape, device=cuda, generator=g).to(torch.bfloat16)
    out.backward(dout)
    ref.backward(dout.float())
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    for name, a_, r_ in zip(("q", "k", "v", "kv", "sink"), leaves, ref_leaves, strict=True):
        if a_ is None:
            continue
        _close(a_.grad, r_.grad, 3e-2 if name != "sink" else 5e-2)


@pytest.mark.parametrize("B,T,nb,nh,c,m,q_start,vis", [(1, 300, 75, 8, 128, 4, 0, False),
                                                      (2, 512, 256, 64, 128, 2, 0, True),
                                                      (1, 200, 130, 5, 64, 1, 37, False)])
def test_indexer_scores_kernel(cuda, B, T, nb, nh, c, m, q_start, vis):
    """Fused indexer scores vs the fp32 oracle sum_h w_h relu(q_h . k_s), block-causal."""
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.gemm import check_errors, error_word

    torch.manual_seed(0)
    q = torch.randn(B, T, nh * c, device=cuda).to(torch.bfloat16)
    keys = torch.randn(B, nb, c, device=cuda).to(torch.bfloat16)
    w = torch.randn(B, T, nh, device=cuda)
    vb = torch.rand(B, nb, device=cuda) if vis else None
    out = torch.empty(B, T, nb, device=cuda)
    backend.ext().indexer_scores(q, keys, w, vb, m, q_start, out, error_word(cuda))
    torch.cuda.synchronize()
    check_errors(cuda)
    qf = q.float().view(B, T, nh, c)
    head = torch.einsum("bthc,bnc->bthn", qf, keys.float()).clamp(min=0)
    ref = (w.unsqueeze(-1) * head).sum(2)
    if vis:
        ref = ref + 0.5 * vb[:, None, :] * w.sum(-1, keepdim=True)
    qpos = torch.arange(q_start, q_start + T, device=cuda)[:, None]
    ok = torch.arange(nb, device=cuda)[None, :] * m + m - 1 < qpos
    ref = ref.masked_fill(~ok, float("-inf"))
    assert torch.equal(torch.isinf(out), torch.isinf(ref))
    fin = torch.isfinite(ref)
    err = (out[fin] - ref[fin]).abs().max().item()
    assert err <= 1e-3 * ref[fin].abs().max().item() + 1e-3, err


@pytest.mark.parametrize("n,k", [(1024, 512), (300, 16), (64, 100), (2048, 1)])
def test_indexer_select_mask_matches_topk(cuda, n, k):
    """Top-k straight to the selection bitmask equals torch.topk + the bitmask kernel on
    scores without ties (block-causal -inf entries included); with ties at the k-th score
    it keeps exactly k, lowest block index first among the ties."""
    from saint_llm_b200.ops import backend, gemm

    torch.manual_seed(n + k)
    rows = 37
    scores = torch.randn(1, rows, n, device=cuda)
    visible = torch.arange(n, device=cuda)[None, :] <= (torch.arange(rows, device=cuda)[:, None] * n) // rows
    scores = scores.masked_fill(~visible[None], float("-inf"))
    words = (n + 31) // 32
    got = torch.empty(1, rows, words, dtype=torch.int32, device=cuda)
    backend.ext().indexer_select_mask(scores.contiguous(), k, got)
    k_eff = min(k, n)
    vals, ids = scores.topk(k_eff, dim=-1)
    top = torch.where(torch.isfinite(vals), ids, torch.full_like(ids, -1))
    want = torch.empty_like(got)
    backend.ext().csa_select_mask(top.contiguous(), n, want, gemm.error_word(cuda))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # ties: every score equal -> the first k blocks
    flat = torch.zeros(1, 2, n, device=cuda)
    sel = torch.empty(1, 2, words, dtype=torch.int32, device=cuda)
    backend.ext().indexer_select_mask(flat, k, sel)
    bits = torch.stack([(sel.view(-1, words)[:, i // 32] >> (i % 32)) & 1 for i in range(n)], -1)
    assert bits.sum(-1).tolist() == [min(k, n)] * 2 and bits[:, :min(k, n)].all()


@pytest.mark.parametrize("B,T,c,m,bias_dtype", [(2, 512, 128, 4, torch.float32), (1, 1000, 64, 128, torch.float32),
                                                (3, 96, 96, 8, torch.bfloat16)])
def test_compressor_pool_kernel_matches_fp32(cuda, B, T, c, m, bias_dtype):
    """compress_pool_fwd / _bwd against the fp32 eager pooling on strided column slices of one
    projection output (T not a multiple of m leaves a tail that gets zero gradient)."""
    from saint_llm_b200.ops.attention import _PoolFn, _pool_torch

    torch.manual_seed(T + m)
    y = (torch.randn(B, T, 3 * c, device=cuda) * 2).to(torch.bfloat16).requires_grad_()
    bias = (torch.randn(m, c, device=cuda) * 0.5).to(bias_dtype).requires_grad_()
    cb, zb = y[..., c:2 * c], y[..., 2 * c:]
    out = _PoolFn.apply(cb, zb, bias, m)
    yr = y.detach().float().requires_grad_()
    br = bias.detach().float().requires_grad_()
    ref = _pool_torch(yr[..., c:2 * c], yr[..., 2 * c:], br, m)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    g = torch.randn_like(ref)
    out.backward(g)
    ref.backward(g)
    torch.testing.assert_close(y.grad.float(), yr.grad, rtol=2e-2, atol=2e-2)
    tol = 2e-2 if bias_dtype == torch.bfloat16 else 1e-3
    torch.testing.assert_close(bias.grad.float(), br.grad, rtol=tol, atol=tol * max(1.0, br.grad.abs().max().item()))

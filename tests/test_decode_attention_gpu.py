"""Native single-token decode attention (one kernel per layer) against the eager
composition of the same step, for SWA, HCA and CSA layers with random caches."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fill(st, gen):
    for t in [st.k, st.v] + ([st.kv.cb, st.kv.zb, st.kv.entries] if st.kv is not None else []) + \
             ([st.idx.cb, st.idx.zb, st.idx.entries] if st.idx is not None else []):
        t.copy_(torch.randn(t.shape, generator=gen).to(t.device, t.dtype))


def _state(st):
    ts = [st.k, st.v]
    for r in (st.kv, st.idx):
        if r is not None:
            ts += [r.cb, r.zb, r.entries]
    return ts


@pytest.mark.parametrize("pos_val", [3, 130, 517])
def test_decode_attention_matches_eager(cuda, pos_val):
    from saint_llm_b200.config import AttentionConfig, CSAConfig, ModelConfig
    from saint_llm_b200.infer.static_decode import StaticDecoder, _attend_layer, _attend_layer_eager
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.models.attention.common import rope_tables

    base = ModelConfig.tiny()
    att = AttentionConfig(**{**base.attention.model_dump(), "query_heads": 8, "head_dim": 128})
    csa = CSAConfig(**{**base.csa.model_dump(), "attention_top_k": 16})
    cfg = base.model_copy(update={"attention": att, "csa": csa, "n_layers": 4})
    torch.manual_seed(0)
    model = SaintLLM(cfg).to(cuda).to(torch.bfloat16).eval()
    with torch.no_grad():
        for blk in model.blocks:
            if blk.attention.sink_logit is not None:
                blk.attention.sink_logit.normal_()
    dec = StaticDecoder(model, 3, 640)
    gen = torch.Generator().manual_seed(1)
    pos = torch.tensor(pos_val, dtype=torch.long, device=cuda)
    cos, sin = rope_tables(640, cfg.attention.rope_dim, cfg.attention.rope_theta, cuda)
    cos, sin = cos[pos_val:pos_val + 1], sin[pos_val:pos_val + 1]
    kinds = set()
    with torch.no_grad():
        for st in dec.layers:
            kinds.add(type(st.attn).__name__)
            _fill(st, gen)
            h = torch.randn(3, 1, cfg.hidden_dim, generator=gen).to(cuda, torch.bfloat16)
            saved = [t.clone() for t in _state(st)]
            got = _attend_layer(st, h, pos, cos, sin)
            after_native = [t.clone() for t in _state(st)]
            for t, s in zip(_state(st), saved, strict=True):
                t.copy_(s)
            want = _attend_layer_eager(st, h, pos, cos, sin)
            torch.cuda.synchronize()
            for a, b in zip(after_native, _state(st), strict=True):
                assert torch.equal(a, b)  # identical cache updates
            err = (got.float() - want.float()).abs().max().item()
            assert err <= 3e-2 * want.float().abs().max().item() + 1e-3, (type(st.attn).__name__, err)
    assert {"CSA", "HCA"} <= kinds


def _pages(rows_per_seq, page_rows, n_pages, gen, cuda):
    """Scatter each sequence's rows into shuffled pages of one pool: (pool, table, lengths)."""
    B = len(rows_per_seq)
    pool = torch.zeros(n_pages, page_rows, 128, dtype=torch.bfloat16)
    perm = torch.randperm(n_pages, generator=gen).tolist()
    maxp = max(1, max((x.shape[0] + page_rows - 1) // page_rows for x in rows_per_seq))
    table = torch.full((B, maxp), -1, dtype=torch.int32)
    for b, x in enumerate(rows_per_seq):
        for p in range((x.shape[0] + page_rows - 1) // page_rows):
            pid = perm.pop()
            table[b, p] = pid
            chunk = x[p * page_rows:(p + 1) * page_rows]
            pool[pid, :chunk.shape[0]] = chunk
    lens = torch.tensor([x.shape[0] for x in rows_per_seq], dtype=torch.int32)
    return pool.to(cuda), table.to(cuda), lens.to(cuda)


@pytest.mark.parametrize("window,softcap,sink", [(0, None, True), (64, 30.0, True), (200, None, False)])
def test_paged_decode_window_matches_fp32(cuda, window, softcap, sink):
    """Variable-length sequences over shuffled pages against fp32 attention over the last
    ``window`` rows of each contiguous history (+ sink, softcap)."""
    import math

    from saint_llm_b200.ops.decode import decode_attention_paged

    gen = torch.Generator().manual_seed(window)
    lens = [1, 37, 300, 129, 64]
    H, P = 8, 16
    ks = [torch.randn(n, 128, generator=gen).to(torch.bfloat16) for n in lens]
    vs = [torch.randn(n, 128, generator=gen).to(torch.bfloat16) for n in lens]
    kp, table, kl = _pages(ks, P, 64, torch.Generator().manual_seed(5), cuda)
    vp, table_v, _ = _pages(vs, P, 64, torch.Generator().manual_seed(5), cuda)
    assert torch.equal(table, table_v)
    q = torch.randn(len(lens), H, 128, generator=gen).to(cuda, torch.bfloat16)
    sk = torch.randn(H, generator=gen).to(cuda) if sink else None
    out = decode_attention_paged(q, kp, vp, table, kl, window=window, sink=sk, softcap=softcap)
    for b, n in enumerate(lens):
        lo = max(0, n - window) if window else 0
        k, v = ks[b][lo:].to(cuda).float(), vs[b][lo:].to(cuda).float()
        s = q[b].float() @ k.t() / math.sqrt(128)
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        if sk is not None:
            s = torch.cat([s, sk[:, None].float()], -1)
        p = torch.softmax(s, -1)[:, :k.shape[0]]
        want = p @ v
        torch.testing.assert_close(out[b].float(), want, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("mode", [1, 2])
def test_paged_decode_compressed_matches_contiguous_kernel(cuda, mode):
    """Same caches laid out as ring + contiguous entries (decode_attention) and as pages
    (decode_attention_paged), all sequences at one position."""
    from saint_llm_b200.ops.decode import decode_attention, decode_attention_paged
    from saint_llm_b200.ops.gemm import check_errors

    gen = torch.Generator().manual_seed(mode)
    B, H, W, m, pos = 3, 8, 128, 4, 517
    n = 160
    kh = torch.randn(B, pos + 1, 128, generator=gen).to(torch.bfloat16)
    vh = torch.randn(B, pos + 1, 128, generator=gen).to(torch.bfloat16)
    ring_k = torch.zeros(B, W, 128, dtype=torch.bfloat16)
    ring_v = torch.zeros(B, W, 128, dtype=torch.bfloat16)
    for r in range(max(0, pos - W + 1), pos + 1):
        ring_k[:, r % W] = kh[:, r]
        ring_v[:, r % W] = vh[:, r]
    ent = torch.randn(B, n, 128, generator=gen).to(torch.bfloat16)
    ne = (pos + 1) // m if mode == 1 else n
    q = torch.randn(B, H, 1, 128, generator=gen).to(cuda, torch.bfloat16)
    sink = torch.randn(H, generator=gen).to(cuda)
    csink = torch.randn(H, generator=gen).to(cuda) if mode == 1 else None
    w = (1 + 0.1 * torch.randn(128, generator=gen)).to(cuda)
    top = torch.randint(-1, ne, (B, 24), generator=gen).to(cuda) if mode == 2 else None
    want = decode_attention(q, ring_k.to(cuda), ring_v.to(cuda), torch.tensor(pos, device=cuda), sink=sink,
                            softcap=None, mode=mode, entries=ent[:, :ne].contiguous().to(cuda), norm_weight=w,
                            m=m, top=top, comp_sink=csink)
    kp, kt, kl = _pages([kh[b] for b in range(B)], 32, 64, torch.Generator().manual_seed(7), cuda)
    vp, _, _ = _pages([vh[b] for b in range(B)], 32, 64, torch.Generator().manual_seed(7), cuda)
    ep, et, el = _pages([ent[b, :ne] for b in range(B)], 32, 32, torch.Generator().manual_seed(8), cuda)
    got = decode_attention_paged(q, kp, vp, kt, kl, window=W, sink=sink, mode=mode, e_pool=ep, e_table=et,
                                 e_len=el, norm_weight=w, m=m, top=top, comp_sink=csink)
    torch.cuda.synchronize()
    check_errors(cuda)
    torch.testing.assert_close(got.float(), want.reshape(B, H, 128).float(), rtol=2e-2, atol=2e-2)


def test_lse_merge_matches_eager_merge(cuda):
    """The one-kernel merge of attention partials against the eager associative merge (tree
    attention's), with empty partials and an extra sink logit."""
    from saint_llm_b200.models.attention.tree import attention_partial, merge_partials
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.decode import lse_merge

    torch.manual_seed(0)
    q = torch.randn(2, 4, 5, 64, device=cuda)
    k = torch.randn(2, 4, 90, 64, device=cuda)
    v = torch.randn(2, 4, 90, 64, device=cuda)
    mask = torch.ones(5, 90, dtype=torch.bool, device=cuda)
    mask[:, 30:60] = False  # the middle chunk is empty for every row
    parts = [attention_partial(q, k[..., s:s + 30, :], v[..., s:s + 30, :], mask[:, s:s + 30]) for s in (0, 30, 60)]
    with backend.eager_mode():
        m0, l0, o0 = merge_partials(parts)
    m1, l1, o1 = lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                           torch.stack([p[2] for p in parts]))
    torch.testing.assert_close(o1, o0, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(l1, l0, rtol=1e-4, atol=1e-4)
    full = torch.softmax((q @ k.transpose(-1, -2) / 8).masked_fill(~mask, float("-inf")), -1) @ v
    torch.testing.assert_close(o1, full, rtol=1e-3, atol=1e-3)
    # a sink joins the denominator only
    sink = torch.randn(4, device=cuda)
    _, _, o2 = lse_merge(torch.stack([p[0] for p in parts]).reshape(3, -1), torch.stack([p[1] for p in parts]).reshape(3, -1),
                         torch.stack([p[2] for p in parts]).reshape(3, -1, 64),
                         extra=sink.repeat_interleave(5).contiguous())
    s = (q @ k.transpose(-1, -2) / 8).masked_fill(~mask, float("-inf"))
    s = torch.cat([s, sink.view(1, 4, 1, 1).expand(2, 4, 5, 1)], -1)
    want = torch.softmax(s, -1)[..., :90] @ v
    torch.testing.assert_close(o2.view(2, 4, 5, 64), want, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("mode,window", [(0, 0), (0, 64), (1, 128), (2, 128)])
def test_paged_decode_split_matches_single_pass(cuda, mode, window):
    from saint_llm_b200.ops.decode import decode_attention_paged
    from saint_llm_b200.ops.gemm import check_errors

    gen = torch.Generator().manual_seed(10 + mode)
    lens = [700, 1, 513, 64]
    H, P, m = 8, 32, 4
    ks = [torch.randn(n, 128, generator=gen).to(torch.bfloat16) for n in lens]
    vs = [torch.randn(n, 128, generator=gen).to(torch.bfloat16) for n in lens]
    kp, kt, kl = _pages(ks, P, 128, torch.Generator().manual_seed(3), cuda)
    vp, _, _ = _pages(vs, P, 128, torch.Generator().manual_seed(3), cuda)
    q = torch.randn(len(lens), H, 128, generator=gen).to(cuda, torch.bfloat16)
    kw = {"window": window, "sink": torch.randn(H, generator=gen).to(cuda), "softcap": 30.0}
    if mode:
        ne = [max(1, n // m) for n in lens]
        ents = [torch.randn(x, 128, generator=gen).to(torch.bfloat16) for x in ne]
        ep, et, el = _pages(ents, P, 64, torch.Generator().manual_seed(4), cuda)
        kw.update(mode=mode, e_pool=ep, e_table=et, e_len=el, norm_weight=torch.ones(128, device=cuda), m=m)
        if mode == 1:
            kw["comp_sink"] = torch.randn(H, generator=gen).to(cuda)
        else:
            kw["top"] = torch.randint(-1, min(ne), (len(lens), 16), generator=gen).to(cuda)
    one = decode_attention_paged(q, kp, vp, kt, kl, **kw)
    four = decode_attention_paged(q, kp, vp, kt, kl, splits=4, **kw)
    torch.cuda.synchronize()
    check_errors(cuda)
    torch.testing.assert_close(four.float(), one.float(), rtol=2e-2, atol=2e-2)

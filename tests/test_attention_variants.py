"""NSA, tree attention (local chunks and 2 gloo ranks) and batch-invariant attention,
against the unmodified reference modules where installed and against dense oracles."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from saint_llm_b200.config import AttentionConfig
from saint_llm_b200.models.attention import (
    NSAttention,
    batch_invariant_attention,
    deterministic_mode,
    tree_attention,
    tree_attention_distributed,
)

ATTN = dict(query_heads=4, head_dim=16, query_compression_dim=24, output_proj_groups=2,
            attention_intermediate_dim=16, sliding_window_size=8, rope_dim=8, use_attention_sink=True)


def _nsa_pair(ref_pkgs, **kw):
    from saint_llm_core.attention.nsa import NSAttention as RefNSA
    from saint_llm_core.config import AttentionConfig as RefAC

    torch.manual_seed(0)
    ref = RefNSA(32, RefAC(**ATTN, **kw), compression_rate=4, selection_k=2)
    ours = NSAttention(32, AttentionConfig(**ATTN, **kw), compression_rate=4, selection_k=2)
    ours.load_state_dict(ref.state_dict())
    with torch.no_grad():  # non-trivial gates and sink
        for m in (ref, ours):
            torch.manual_seed(1)
            m.branch_gate.weight.normal_(0, 0.3)
            m.sink_logit.normal_()
    return ref, ours


@pytest.mark.parametrize("softcap", [None, 5.0])
def test_nsa_matches_reference(ref_pkgs, softcap):
    ref, ours = _nsa_pair(ref_pkgs, logit_softcap=softcap)
    assert sorted(ref.state_dict()) == sorted(ours.state_dict())
    h = torch.randn(2, 21, 32)
    h1, h2 = h.clone().requires_grad_(True), h.clone().requires_grad_(True)
    yr, yo = ref(h1), ours(h2)
    torch.testing.assert_close(yo, yr, atol=1e-5, rtol=1e-4)
    assert abs(ours._last_max_attn_logit - ref._last_max_attn_logit) < 1e-4
    yr.square().sum().backward()
    yo.square().sum().backward()
    torch.testing.assert_close(h2.grad, h1.grad, atol=1e-4, rtol=1e-3)
    mine = dict(ours.named_parameters())
    for n, a in ref.named_parameters():
        torch.testing.assert_close(mine[n].grad, a.grad, atol=1e-4, rtol=1e-3, msg=n)


def test_nsa_cached_decode_matches_full():
    from saint_llm_b200.infer.kv_cache import SWAKVCacheLayer

    torch.manual_seed(0)
    m = NSAttention(32, AttentionConfig(**ATTN), compression_rate=4, selection_k=2)
    h = torch.randn(1, 19, 32)
    full = m(h)
    cache = SWAKVCacheLayer(32, 16)
    parts = [m(h[:, :11], kv_cache=cache)] + [m(h[:, t:t + 1], kv_cache=cache) for t in range(11, 19)]
    torch.testing.assert_close(torch.cat(parts, 1), full, atol=1e-5, rtol=1e-4)


def test_nsa_model_pattern_and_cache():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.infer import greedy_decode, greedy_decode_cached
    from saint_llm_b200.models import SaintLLM

    cfg = ModelConfig.tiny().model_copy(update={"attention_pattern": "nsa"})
    torch.manual_seed(0)
    model = SaintLLM(cfg).eval()
    assert isinstance(model.blocks[-1].attention, NSAttention)
    x = torch.randint(0, cfg.vocab_size, (1, 9))
    assert torch.equal(greedy_decode(model, x, max_new_tokens=4), greedy_decode_cached(model, x, max_new_tokens=4))


def _dense(q, k, v, mask):
    s = (q @ k.transpose(-1, -2)) / q.shape[-1] ** 0.5
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), -1).nan_to_num(0.0)
    return p @ v


@pytest.mark.parametrize("n_chunks", [1, 3, 4, 7])
def test_tree_attention_matches_dense(n_chunks):
    torch.manual_seed(0)
    q, k, v = torch.randn(2, 3, 10, 8), torch.randn(2, 3, 12, 8), torch.randn(2, 3, 12, 8)
    mask = torch.ones(10, 12, dtype=torch.bool).tril(2)
    mask[0] = False  # a row that sees nothing outputs zero
    out = tree_attention(q, k, v, n_chunks=n_chunks, mask=mask)
    torch.testing.assert_close(out, _dense(q, k, v, mask), atol=1e-5, rtol=1e-5)
    with pytest.raises(ValueError):
        tree_attention(q, k, v, n_chunks=0)


def test_tree_attention_matches_reference(ref_pkgs):
    from saint_llm_core.attention.tree_attention import tree_attention as ref_tree

    torch.manual_seed(1)
    q, k, v = torch.randn(1, 2, 9, 8), torch.randn(1, 2, 9, 8), torch.randn(1, 2, 9, 8)
    mask = torch.ones(9, 9, dtype=torch.bool).tril()
    torch.testing.assert_close(tree_attention(q, k, v, n_chunks=3, mask=mask),
                               ref_tree(q, k, v, n_chunks=3, mask=mask), atol=1e-5, rtol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tree_worker(rank, ws, port, q_out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        torch.manual_seed(0)
        q, k, v = torch.randn(1, 2, 6, 8), torch.randn(1, 2, 10, 8), torch.randn(1, 2, 10, 8)
        mask = torch.ones(6, 10, dtype=torch.bool).tril(4)
        sl = slice(rank * 5, rank * 5 + 5)
        out = tree_attention_distributed(q, k[:, :, sl], v[:, :, sl], mask_local=mask[:, sl])
        q_out.put((rank, bool(torch.allclose(out, _dense(q, k, v, mask), atol=1e-5))))
    finally:
        dist.destroy_process_group()


@pytest.mark.distributed
def test_tree_attention_two_ranks():
    ctx = mp.get_context("spawn")
    q, port = ctx.Queue(), _free_port()
    ps = [ctx.Process(target=_tree_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res


def test_batch_invariant_attention():
    torch.manual_seed(0)
    q, k, v = torch.randn(4, 2, 5, 8), torch.randn(4, 2, 7, 8), torch.randn(4, 2, 7, 8)
    full = batch_invariant_attention(q, k, v, is_causal=True)
    one = batch_invariant_attention(q[2:3], k[2:3], v[2:3], is_causal=True)
    assert torch.equal(full[2:3], one)
    torch.testing.assert_close(full, F.scaled_dot_product_attention(q, k, v, attn_mask=torch.ones(5, 7).bool()
                                                                     .tril(2)), atol=1e-5, rtol=1e-5)
    m = torch.zeros(5, 7, dtype=torch.bool)
    assert float(batch_invariant_attention(q, k, v, attn_mask=m).abs().max()) == 0.0


def test_deterministic_mode_restores_state():
    before = (torch.are_deterministic_algorithms_enabled(), os.environ.get("CUBLAS_WORKSPACE_CONFIG"))
    with pytest.raises(RuntimeError):
        with deterministic_mode():
            assert torch.are_deterministic_algorithms_enabled()
            assert os.environ["CUBLAS_WORKSPACE_CONFIG"]
            raise RuntimeError("body")
    assert (torch.are_deterministic_algorithms_enabled(), os.environ.get("CUBLAS_WORKSPACE_CONFIG")) == before

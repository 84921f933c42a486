"""CPU checks of components with no other direct test: MTP heads, the NSA selective branch
against a per-query loop, agent memory stores and tools, tokenizer fertility and the GRPO
response mask."""

from __future__ import annotations

import math

import pytest
import torch

from saint_llm_b200.agents.core import ToolCall, ToolRegistry
from saint_llm_b200.agents.memory import (FileMemoryStore, InMemoryMemoryStore, memory_tools,
                                          register_memory_tools)
from saint_llm_b200.config import MTPConfig
from saint_llm_b200.data.fertility import measure_fertility, measure_per_language_fertility
from saint_llm_b200.data.tokenizer import CharTokenizer
from saint_llm_b200.models.attention.nsa import block_compress, selective_attention
from saint_llm_b200.models.mtp import MTPStack, shift_left
from saint_llm_b200.posttrain.rollout import response_mask_through_eos


# ----------------------------------------------------------------------------- MTP
def test_shift_left_pads_with_zeros_at_the_end():
    x = torch.arange(12, dtype=torch.float32).view(1, 4, 3)
    y = shift_left(x, 1)
    assert torch.equal(y[:, :3], x[:, 1:]) and torch.equal(y[:, 3], torch.zeros(1, 3))
    assert torch.equal(shift_left(x, 4), torch.zeros_like(x))
    assert torch.equal(shift_left(x, 9), torch.zeros_like(x))


def test_mtp_stack_chains_depths_and_backpropagates():
    torch.manual_seed(0)
    d, depth = 16, 3
    stack = MTPStack(d, 100, MTPConfig(depth=depth))
    h = torch.randn(2, 6, d, requires_grad=True)
    e = torch.randn(2, 6, d, requires_grad=True)
    outs = stack(h, e)
    assert len(outs) == depth and all(o.shape == h.shape for o in outs)
    # depth k is module k applied to depth k-1's output and the embeddings shifted by k+1
    cur = h
    for k, mod in enumerate(stack.modules_):
        cur = mod(cur, shift_left(e, k + 1))
        torch.testing.assert_close(outs[k], cur)
    sum(o.square().mean() for o in outs).backward()
    assert h.grad is not None and h.grad.abs().sum() > 0
    # every depth shifts by at least one: position 0's embedding is never read
    assert torch.count_nonzero(e.grad[:, 0]) == 0 and torch.count_nonzero(e.grad[:, 1]) > 0
    stack.zero_grad()
    e.grad = None
    stack(h, e)[0][:, -1].sum().backward()
    assert torch.count_nonzero(e.grad) == 0  # position T-1 of depth 0 reads the zero padding


# ----------------------------------------------------------------------------- NSA
def test_block_compress_means_and_drops_the_tail():
    x = torch.arange(2 * 10 * 3, dtype=torch.float32).view(2, 10, 3)
    y = block_compress(x, block_size=4)
    assert y.shape == (2, 2, 3)
    torch.testing.assert_close(y[:, 1], x[:, 4:8].mean(1))
    assert block_compress(x, block_size=16).shape == (2, 0, 3)
    assert block_compress(x, block_size=0).shape == (2, 0, 3)


def _selective_loop(q, k, v, block_size, top_k, q_start, softcap):
    """Per (b, h, t): score the visible pooled blocks, keep the top_k, attend over their tokens."""
    b, h, tq, d = q.shape
    nb = k.shape[1] // block_size
    out = torch.zeros_like(q)
    kc = block_compress(k, block_size=block_size)
    for bi in range(b):
        for hi in range(h):
            for t in range(tq):
                pos = q_start + t
                vis = [i for i in range(nb) if (i + 1) * block_size - 1 <= pos]
                if not vis:
                    continue
                s = torch.stack([q[bi, hi, t] @ kc[bi, i] for i in vis]) / math.sqrt(d)
                picked = [vis[j] for j in s.topk(min(top_k, len(vis))).indices.tolist()]
                toks = torch.cat([torch.arange(i * block_size, (i + 1) * block_size) for i in sorted(picked)])
                sc = k[bi, toks] @ q[bi, hi, t] / math.sqrt(d)
                if softcap is not None:
                    sc = softcap * torch.tanh(sc / softcap)
                out[bi, hi, t] = torch.softmax(sc, 0) @ v[bi, toks]
    return out


@pytest.mark.parametrize("q_start,softcap,top_k", [(0, None, 2), (5, 30.0, 1), (0, None, 10)])
def test_selective_attention_matches_a_per_query_loop(q_start, softcap, top_k):
    torch.manual_seed(1)
    b, h, tq, d, m = 2, 2, 12, 8, 4
    tk = q_start + tq
    q = torch.randn(b, h, tq, d, dtype=torch.float64)
    k = torch.randn(b, tk, d, dtype=torch.float64)
    v = torch.randn(b, tk, d, dtype=torch.float64)
    got = selective_attention(q, k, v, block_size=m, top_k=top_k, q_start=q_start, logit_softcap=softcap,
                              query_chunk=5)
    want = _selective_loop(q, k, v, m, top_k, q_start, softcap)
    torch.testing.assert_close(got, want)
    if q_start == 0:  # queries before the first complete block see nothing
        assert torch.count_nonzero(got[:, :, : m - 1]) == 0


def test_selective_attention_without_blocks_is_zero():
    q = torch.randn(1, 1, 3, 4)
    k = v = torch.randn(1, 3, 4)
    assert torch.count_nonzero(selective_attention(q, k, v, block_size=4, top_k=2)) == 0
    k = v = torch.randn(1, 8, 4)
    assert torch.count_nonzero(selective_attention(q, k, v, block_size=4, top_k=0)) == 0


# -------------------------------------------------------------------------- memory
@pytest.mark.parametrize("kind", ["memory", "file"])
def test_memory_store_contract(kind, tmp_path, monkeypatch):
    clock = iter(float(i) for i in range(100))
    monkeypatch.setattr("saint_llm_b200.agents.memory.time.time", lambda: next(clock))
    store = InMemoryMemoryStore() if kind == "memory" else FileMemoryStore(tmp_path / "mem")
    store.store("alpha", "the first note")
    store.store("beta.v2", "Second NOTE\nwith two lines")
    store.store("gamma_3", "unrelated")
    assert store.view("alpha").value == "the first note"
    assert store.view("missing") is None
    assert [e.key for e in store.list()] == ["gamma_3", "beta.v2", "alpha"]  # newest first
    assert [e.key for e in store.recall("note")] == ["beta.v2", "alpha"]      # case-insensitive
    assert [e.key for e in store.recall("note", limit=1)] == ["beta.v2"]
    assert store.recall("") == ()
    assert [e.key for e in store.recall("GAMMA")] == ["gamma_3"]             # key match
    store.store("alpha", "rewritten")
    assert store.view("alpha").value == "rewritten" and store.list()[0].key == "alpha"
    assert store.delete("alpha") is True and store.delete("alpha") is False
    for bad in ("", ".", "..", "a/b", "sp ace", "../x"):
        with pytest.raises(ValueError):
            store.store(bad, "x")
    store.clear()
    assert store.list() == ()


def test_file_memory_store_persists_and_ignores_foreign_files(tmp_path):
    root = tmp_path / "mem"
    FileMemoryStore(root).store("k1", "v1")
    (root / "notes.txt").write_text("not an entry")
    (root / "k2.meta").write_text("{broken")
    (root / "k2.md").write_text("v2")
    again = FileMemoryStore(root)
    assert again.view("k1").value == "v1"
    assert again.view("k2").created_at == 0.0  # unreadable timestamp falls back to 0
    assert {e.key for e in again.list()} == {"k1", "k2"}
    again.clear()
    assert (root / "notes.txt").exists() and again.list() == ()


def test_memory_tools_through_a_registry():
    store = InMemoryMemoryStore()
    reg = ToolRegistry()
    register_memory_tools(reg, store, name_prefix="m_")
    assert {s.name for s in reg.specs()} == {"m_view", "m_store", "m_recall", "m_delete"}
    assert reg.execute(ToolCall("1", "m_store", {"key": "city", "value": "Kyiv\nUkraine"})).content == "ok"
    assert reg.execute(ToolCall("2", "m_view", {"key": "city"})).content == "Kyiv\nUkraine"
    assert reg.execute(ToolCall("3", "m_recall", {"query": "kyiv"})).content == "city: Kyiv Ukraine"
    assert reg.execute(ToolCall("4", "m_delete", {"key": "city"})).content == "deleted"
    assert reg.execute(ToolCall("5", "m_view", {"key": "city"})).content == "no entry"
    err = reg.execute(ToolCall("6", "m_store", {"key": "bad key", "value": "x"}))
    assert err.content.startswith("ERROR: ValueError") and err.tool_call_id == "6"
    specs = {t.spec.name: t.spec for t in memory_tools(store)}
    assert specs["memory_store"].parameters["required"] == ["key", "value"]


# ------------------------------------------------------------------------ fertility
def test_fertility_per_language():
    tok = CharTokenizer()
    assert measure_fertility(tok, "") == (0, 0)
    assert measure_fertility(tok, "héllo") == (5, 5)
    rep = measure_per_language_fertility(tok, {"uk": ["привіт", "світ"], "en": ["hi"], "empty": ["", ""]})
    by = rep.by_language()
    assert list(by) == ["en", "uk"]  # sorted, languages without characters dropped
    assert by["uk"].n_samples == 2 and by["uk"].chars == 10 and by["uk"].fertility == 1.0
    assert rep.to_dict()["records"][0]["language"] == "en"


# --------------------------------------------------------------------- response mask
def test_response_mask_through_first_eos():
    toks = torch.tensor([[5, 6, 7, 1, 8, 1],
                         [5, 6, 1, 9, 9, 9],
                         [5, 6, 7, 8, 9, 9]])
    m = response_mask_through_eos(toks, 2, eos=1)
    assert m.tolist() == [[0, 0, 1, 1, 0, 0],
                          [0, 0, 1, 0, 0, 0],
                          [0, 0, 1, 1, 1, 1]]
    assert response_mask_through_eos(toks, 2, eos=None)[:, 2:].all()
    # an EOS inside the prompt does not cut the response
    assert response_mask_through_eos(torch.tensor([[1, 1, 4, 4]]), 2, eos=1).tolist() == [[0, 0, 1, 1]]

"""Paged KV pool: streams of mixed lengths share pages, gathers equal contiguous rows, pages
come back on release / truncate, and attention over block tables equals dense attention."""

import math

import pytest
import torch

from saint_llm_b200.infer.paged_kv import PagedKVManager, PagePool, PagedStream, PoolExhausted, paged_attention


def test_stream_append_gather_truncate_release():
    pool = PagePool(8, 4, 3, dtype=torch.float32)
    s = PagedStream(pool)
    rows = torch.arange(30, dtype=torch.float32).view(10, 3)
    s.append(rows[:3])
    s.append(rows[3:10])
    assert s.length == 10 and len(s.pages) == 3 and pool.free_pages == 5
    assert torch.equal(s.gather(), rows)
    s.truncate(5)
    assert len(s.pages) == 2 and pool.free_pages == 6 and torch.equal(s.gather(), rows[:5])
    s.append(rows[5:7])
    assert torch.equal(s.gather(), rows[:7])
    s.release()
    assert pool.free_pages == 8 and s.length == 0


def test_pool_exhaustion_and_reuse():
    pool = PagePool(2, 2, 1, dtype=torch.float32)
    a, b = PagedStream(pool), PagedStream(pool)
    a.append(torch.ones(4, 1))
    with pytest.raises(PoolExhausted):
        b.append(torch.ones(1, 1))
    a.release()
    b.append(torch.full((3, 1), 2.0))
    assert torch.equal(b.gather(), torch.full((3, 1), 2.0))


def test_manager_mixed_lengths_and_attention():
    torch.manual_seed(0)
    d, h = 16, 4
    pools = {"k": PagePool(64, 8, d, dtype=torch.float32), "v": PagePool(64, 8, d, dtype=torch.float32)}
    mgr = PagedKVManager(pools, n_layers=2)
    lens = {"a": 5, "b": 19, "c": 1}
    ref = {}
    for r, n in lens.items():
        mgr.admit(r)
        k, v = torch.randn(n, d), torch.randn(n, d)
        # append in uneven chunks, interleaved with another request
        mgr.append(r, 1, "k", k[:2]); mgr.append(r, 1, "v", v[:2])
        mgr.append(r, 1, "k", k[2:]); mgr.append(r, 1, "v", v[2:])
        ref[r] = (k, v)
    reqs = ["b", "a", "c"]
    kp, lengths = mgr.gather_padded(reqs, 1, "k")
    assert lengths.tolist() == [19, 5, 1]
    for i, r in enumerate(reqs):
        assert torch.equal(kp[i, :lens[r]], ref[r][0])
    table, lengths = mgr.block_tables(reqs, 1, "k")
    vtable, _ = mgr.block_tables(reqs, 1, "v")
    assert table.shape == (3, 3) and (table[2, 1:] == -1).all()
    q = torch.randn(3, h, d)
    sink = torch.randn(h)
    # K and V pages were allocated in lockstep, so the K table also indexes V
    assert torch.equal(table, vtable)
    out = paged_attention(q, pools["k"], pools["v"], table, lengths, sink=sink)
    for i, r in enumerate(reqs):
        k, v = ref[r]
        s = q[i] @ k.t() / math.sqrt(d)
        s = torch.cat([s, sink[:, None]], dim=-1)
        p = torch.softmax(s, dim=-1)[:, :-1]
        assert torch.allclose(out[i], p @ v, atol=1e-5)
    mgr.release("b")
    assert pools["k"].free_pages == 64 - 1 - 1  # "a" (5 rows) and "c" (1 row): one page each


def test_append_is_all_or_nothing_and_double_free_raises():
    import pytest

    from saint_llm_b200.infer.paged_kv import PagedStream, PagePool, PoolExhausted

    pool = PagePool(3, 4, 2, dtype=torch.float32)
    s = PagedStream(pool)
    s.append(torch.ones(6, 2))  # 2 pages
    before = (list(s.pages), s.length, pool.free_pages)
    with pytest.raises(PoolExhausted):
        s.append(torch.zeros(7, 2))  # needs 2 more pages, 1 free
    assert (list(s.pages), s.length, pool.free_pages) == before
    assert torch.equal(s.gather(), torch.ones(6, 2))
    s.append(torch.full((2, 2), 2.0))  # fills page 2 exactly
    assert s.length == 8 and pool.free_pages == 1
    with pytest.raises(ValueError):
        pool.free([s.pages[0], s.pages[0]])
    s.release()
    with pytest.raises(ValueError):
        pool.free([0])  # already free
    assert pool.free_pages == 3

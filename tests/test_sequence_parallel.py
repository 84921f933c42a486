"""Ulysses and ring attention (contiguous and zigzag sharding) on gloo CPU ranks against
single-process attention: outputs and q / k / v gradients."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.distributed


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, ws, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        q.put(_check(rank, ws))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _check(rank, ws):
    from saint_llm_b200.parallel import sp

    B, T, H, d = 2, 32, 4, 16
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(B, T, H, d, generator=g) for _ in range(3))
    dy = torch.randn(B, T, H, d, generator=g)
    results = []
    for shard in ("contiguous", "zigzag"):
        pos = (sp.zigzag_positions if shard == "zigzag" else sp.contiguous_positions)(T, rank, ws)
        for fn in (sp.ulysses_attention, sp.ring_attention):
            for causal, window in ((True, None), (True, 7), (False, None)):
                qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
                ref = sp.local_attention(qf, kf, vf, torch.arange(T), torch.arange(T), causal=causal, window=window)
                (ref * dy).sum().backward()
                ql, kl, vl = (t[:, pos].clone().requires_grad_(True) for t in (q, k, v))
                out = fn(ql, kl, vl, pos, causal=causal, window=window)
                (out * dy[:, pos]).sum().backward()
                ok = torch.allclose(out, ref[:, pos], atol=1e-5, rtol=1e-4)
                for a, b in ((ql, qf), (kl, kf), (vl, vf)):
                    ok = ok and torch.allclose(a.grad, b.grad[:, pos], atol=1e-5, rtol=1e-4)
                results.append((shard, fn.__name__, causal, window, ok))
    return rank, all(r[-1] for r in results), [r for r in results if not r[-1]]


@pytest.mark.parametrize("ws", [2, 4])
def test_ulysses_and_ring_attention_match_single_process(ws):
    ctx = mp.get_context("spawn")
    q, port = ctx.Queue(), _port()
    ps = [ctx.Process(target=_entry, args=(r, ws, port, q)) for r in range(ws)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(ws)]
    for p in ps:
        p.join(timeout=60)
    for r in res:
        assert r[1] is True, r


@pytest.mark.parametrize("ws", [1, 2, 4, 8])
def test_sharding_positions_partition_the_sequence(ws):
    """Every token lands on exactly one rank; zigzag pairs an early chunk with a late one, so
    each rank's causal work (sum of query positions + 1) is the same."""
    from saint_llm_b200.parallel import sp

    T = 64
    for fn in (sp.contiguous_positions, sp.zigzag_positions):
        parts = [fn(T, r, ws) for r in range(ws)]
        allpos = torch.cat(parts).sort().values
        assert torch.equal(allpos, torch.arange(T)), fn.__name__
        assert all(p.numel() == T // ws for p in parts)
    work = [int((sp.zigzag_positions(T, r, ws) + 1).sum()) for r in range(ws)]
    assert max(work) == min(work)

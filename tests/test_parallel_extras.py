"""Distributed-training building blocks: ZeRO planner and owner-partitioned sync (2 gloo
ranks), DiLoCo / NoLoCo outer loops, ring all-reduce simulation, gradient compression,
peer verification / reputation / decentralised rounds, the miner/validator protocol and
FSDP2 wrapping."""

import os
import socket
import threading

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from saint_llm_b200.parallel import bittensor as bt
from saint_llm_b200.parallel import compression as gc
from saint_llm_b200.parallel import local_sgd as ls
from saint_llm_b200.parallel import trust
from saint_llm_b200.parallel import zero


def _tiny() -> nn.Module:
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(8, 4, bias=False), nn.Linear(4, 2, bias=False))


# ------------------------------------------------------------------ ZeRO planner
def test_lpt_packing_balances():
    a = zero.pack_buckets_by_cost([4.0, 3.0, 2.0, 1.0], 2)
    assert a.per_rank_cost == (5.0, 5.0)
    assert zero.pack_buckets_by_cost([10.0, 1.0, 1.0, 1.0], 2).imbalance == pytest.approx(0.7)
    assert zero.pack_buckets_by_cost([], 3).imbalance == 0.0
    assert sum(len(b) for b in zero.pack_buckets_by_cost([0.0] * 3, 2).buckets) == 3
    with pytest.raises(ValueError):
        zero.pack_buckets_by_cost([1.0], 0)
    with pytest.raises(ValueError):
        zero.pack_buckets_by_cost([-1.0], 2)


def test_hybrid_assign_splits_pools():
    ps = [torch.zeros(100, 100), torch.zeros(100, 100), torch.zeros(1000), torch.zeros(1000)]
    a = zero.hybrid_zero_assign(ps, ["muon", "muon", "adamw", "adamw"], 2)
    assert a.per_rank_cost == (11000.0, 11000.0)
    owner = a.owner_of()
    assert sorted(owner) == [0, 1, 2, 3]
    assert owner[0] != owner[1] and owner[2] != owner[3]
    assert zero.muon_param_cost(torch.zeros(2, 4, 8)) == 64
    with pytest.raises(ValueError):
        zero.hybrid_zero_assign([torch.zeros(2)], ["lion"], 2)
    with pytest.raises(ValueError):
        zero.hybrid_zero_assign([torch.zeros(2)], ["muon", "adamw"], 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _zero_worker(rank: int, ws: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.optim.muon import MuonAdamW

        model = _tiny()
        params = list(model.parameters())
        sync = zero.ZeroOptimizerSync(params, ["muon", "adamw"], bucket_bytes=16)
        torch.manual_seed(10 + rank)
        x = torch.randn(5, 8)
        model(x).square().sum().backward()
        grads = [p.grad.clone() for p in params]
        mean = [g.clone() for g in grads]
        for g in mean:
            dist.all_reduce(g)
            g /= ws
        sync.reduce_grads()
        ok_grad = all(torch.allclose(p.grad, m, atol=1e-6) if sync.is_owned(p) else bool((p.grad == 0).all())
                      for p, m in zip(params, mean, strict=True))
        # reference update: full optimizer on the mean gradient on every rank
        ref = _tiny()
        for p, m in zip(ref.parameters(), mean, strict=True):
            p.grad = m.clone()
        ref_opt = MuonAdamW([ref[0].weight], [ref[1].weight], lr=0.01, adamw_lr=0.01)
        ref_opt.step()
        opt = MuonAdamW([model[0].weight], [model[1].weight], lr=0.01, adamw_lr=0.01)
        opt.param_filter = sync.is_owned
        opt.step()
        sync.broadcast_params()
        ok_step = all(torch.allclose(a, b, atol=1e-6) for a, b in zip(model.parameters(), ref.parameters(),
                                                                        strict=True))
        q.put((rank, ok_grad, ok_step, len(sync.owned)))
    finally:
        dist.destroy_process_group()


@pytest.mark.distributed
def test_zero_sync_two_ranks_matches_replicated_step():
    ctx = mp.get_context("spawn")
    q, port = ctx.Queue(), _free_port()
    procs = [ctx.Process(target=_zero_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(g and s for _, g, s, _ in res), res
    assert sum(n for *_, n in res) == 2


# ------------------------------------------------------------------ DiLoCo / NoLoCo
def test_diloco_outer_update_matches_nesterov_formula():
    m = _tiny()
    cfg = ls.DiLoCoConfig(inner_steps=2, outer_lr=0.5, outer_momentum=0.9, nesterov=True)
    d = ls.DiLoCo(m.parameters(), cfg)
    snap = [p.detach().clone() for p in m.parameters()]
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.1)
    d.inner_step()
    assert not d.should_sync
    d.inner_step()
    assert d.should_sync
    d.outer_sync()
    assert not d.should_sync
    for p, s in zip(m.parameters(), snap, strict=True):
        g = torch.full_like(s, -0.1)
        torch.testing.assert_close(p.detach(), s - 0.5 * (g + 0.9 * g))
    st = d.state_dict()
    d2 = ls.DiLoCo(m.parameters(), cfg)
    d2.load_state_dict(st)
    assert torch.equal(d2.state_dict()["momentum_buffer"][0], st["momentum_buffer"][0])


def test_diloco_reducer_scales_update():
    class Half:
        def reduce(self, ts):
            return [t * 0.5 for t in ts]

    m = _tiny()
    d = ls.DiLoCo(m.parameters(), ls.DiLoCoConfig(inner_steps=1, outer_lr=1.0, outer_momentum=0.0), reducer=Half())
    snap = [p.detach().clone() for p in m.parameters()]
    with torch.no_grad():
        for p in m.parameters():
            p.add_(1.0)
    d.inner_step()
    d.outer_sync()
    for p, s in zip(m.parameters(), snap, strict=True):
        torch.testing.assert_close(p.detach(), s + 0.5)


def test_ring_all_reduce_and_threads():
    assert [ls.ring_log2_rounds(n) for n in (0, 1, 2, 3, 4, 7, 8)] == [0, 0, 1, 2, 2, 3, 3]
    ins = [[torch.tensor([float(i), 2.0 * i])] for i in range(4)]
    out = ls.ring_all_reduce(ins)
    for o in out:
        torch.testing.assert_close(o[0], torch.tensor([1.5, 3.0]))
    sim = ls.RingAllReduceSimulator(4)
    res = [None] * 4

    def run(i):
        res[i] = sim.peer_reducer(i).reduce([torch.tensor([float(i)])])

    th = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=10)
    assert all(torch.allclose(r[0], torch.tensor([1.5])) for r in res)


def test_noloco_adam_outer_step():
    m = _tiny()
    cfg = ls.NoLoCoConfig(inner_steps=1, outer_lr=0.01)
    n = ls.NoLoCo(m.parameters(), cfg, reducer=ls.IdentityReducer())
    snap = [p.detach().clone() for p in m.parameters()]
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.2)
    n.inner_step()
    n.outer_sync()
    # first Adam step moves every coordinate by lr in the sign of -pseudo-gradient
    for p, s in zip(m.parameters(), snap, strict=True):
        torch.testing.assert_close(p.detach(), s + 0.01, atol=1e-6, rtol=0)
    n2 = ls.NoLoCo(m.parameters(), cfg, reducer=ls.IdentityReducer())
    n2.load_state_dict(n.state_dict())
    assert n2.state_dict()["step"] == 1


# ------------------------------------------------------------------ compression
def test_topk_and_residual():
    g = torch.tensor([0.1, -5.0, 0.3, 4.0, -0.2, 0.0])
    c = gc.top_k_compression(g, density=2 / 6)
    assert sorted(c.indices.tolist()) == [1, 3]
    torch.testing.assert_close(gc.decompress(c), torch.tensor([0.0, -5.0, 0.0, 4.0, 0.0, 0.0]))
    comp = gc.TopKWithResidualCompressor(density=1 / 6)
    c1 = comp.step(g)
    c2 = comp.step(torch.zeros(6))
    assert c1.indices.tolist() == [1] and c2.indices.tolist() == [3]  # residual carried over
    with pytest.raises(ValueError):
        gc.top_k_compression(g, density=0.0)


def test_bloom_and_sparse_loco():
    m, k = gc.bloom_size_for(100, 0.01)
    b = gc.SparseLoCoBloom.empty(m_bits=m, n_hashes=k)
    b.add_many(torch.arange(100))
    assert bool(b.contains_many(torch.arange(100)).all())
    fp = b.contains_many(torch.arange(10_000, 20_000)).float().mean().item()
    assert fp < 0.05
    g = torch.randn(1000)
    c_a, bloom_a = gc.sparse_loco_compress(g, density=0.05)
    c_b, _ = gc.sparse_loco_compress(g, density=0.05, peer_bloom=bloom_a)
    assert len(set(c_a.indices.tolist()) & set(c_b.indices.tolist())) <= 2
    merged = bloom_a.merged_with(gc.SparseLoCoBloom.empty(m_bits=bloom_a.m_bits, n_hashes=bloom_a.n_hashes))
    assert torch.equal(merged.bits, bloom_a.bits)


# ------------------------------------------------------------------ trust
def _mse(model, x, y):
    return (model(x) - y).square().mean()


def _honest(model, x, y):
    model.zero_grad()
    _mse(model, x, y).backward()
    return [p.grad.clone() for p in model.parameters()], [n for n, _ in model.named_parameters()]


def test_verifier_accepts_honest_rejects_random_and_restores_grads():
    m = _tiny()
    x, y = torch.randn(6, 8), torch.randn(6, 2)
    grads, names = _honest(m, x, y)
    marker = [torch.full_like(p, 7.0) for p in m.parameters()]
    for p, g in zip(m.parameters(), marker, strict=True):
        p.grad = g
    v = trust.GradientVerifier(m, _mse)
    assert v.verify(grads, names, inputs=x, labels=y).accepted
    bad, bad_names = trust.random_peer_gradient(m, seed=3)
    r = v.verify(bad, bad_names, inputs=x, labels=y)
    assert not r.accepted and r.reason.startswith("rejected")
    assert all(torch.equal(p.grad, g) for p, g in zip(m.parameters(), marker, strict=True))
    neg = [-g for g in grads]
    assert v.verify(neg, names, inputs=x, labels=y).min_cosine < 0


def test_reputation_ewma_and_weighted_reduce():
    t = trust.PeerReputationTracker(trust.PeerReputationConfig(initial_score=0.5, decay=0.5))
    assert t.update("a", accepted=True) == pytest.approx(0.75)
    assert t.update("b", accepted=False) == pytest.approx(0.25)
    out = trust.reputation_weighted_reduce([[torch.tensor([1.0])], [torch.tensor([5.0])]], ["a", "b"], t)
    torch.testing.assert_close(out[0], torch.tensor([0.75 * 1 + 0.25 * 5.0]))
    out = trust.reputation_weighted_reduce([[torch.tensor([1.0])], [torch.tensor([5.0])]], ["a", "b"], t,
                                           min_score=0.5)
    torch.testing.assert_close(out[0], torch.tensor([1.0]))
    with pytest.raises(ValueError):
        trust.PeerReputationConfig(decay=1.0)


def test_decentralized_round():
    m = _tiny()
    x, y = torch.randn(6, 8), torch.randn(6, 2)
    g, names = _honest(m, x, y)
    bad, _ = trust.random_peer_gradient(m, seed=1)
    tr = trust.PeerReputationTracker()
    rnd = trust.DecentralizedTrainingRound(verifier=trust.GradientVerifier(m, _mse), tracker=tr)
    res = rnd.process([trust.PeerSubmission("h1", g, names, x, y), trust.PeerSubmission("h2", g, names, x, y),
                       trust.PeerSubmission("evil", bad, names, x, y)])
    assert res.n_accepted == 2 and [o.accepted for o in res.outcomes] == [True, True, False]
    torch.testing.assert_close(res.aggregated[0], g[0])
    assert tr.score("evil") < tr.score("h1")


# ------------------------------------------------------------------ miner / validator
class _Echo:
    def __init__(self, text):
        self.text = text

    def serve(self, query):
        return self.text


class _LenScorer:
    def score(self, query, response):
        return float(len(response))


def test_miner_validator_over_channels():
    from saint_llm_b200.agents.jsonrpc import pair_channels

    chans, threads = {}, []
    for uid, text in (("m1", "aa"), ("m2", "aaaa"), ("m3", "")):
        client, server = pair_channels()
        srv = bt.BittensorMinerServer(_Echo(text), bt.MinerInfo(uid, name=uid))
        th = threading.Thread(target=srv.serve, args=(server,), daemon=True)
        th.start()
        chans[uid], threads = client, threads + [th]
    v = bt.BittensorValidatorClient(scorer=_LenScorer(), channels=chans)
    scores = {s.uid: s for s in v.query_and_score("q")}
    assert scores["m1"].weight == pytest.approx(1 / 3) and scores["m2"].weight == pytest.approx(2 / 3)
    assert scores["m3"].raw_score == 0.0
    for c in chans.values():
        c.close()
    assert bt.cohort_consensus_score("q", "the cat", peer_responses=["a cat", "dog"]) == 0.5
    assert bt.aggregate_cohort_scores([1.0, 3.0, 2.0], mode="median") == 2.0
    with pytest.raises(ValueError):
        bt.aggregate_cohort_scores([1.0], mode="sum")


# ------------------------------------------------------------------ FSDP2
def test_fsdp_block_policy():
    from saint_llm_b200.parallel.fsdp import default_block_policy

    class FooBlock(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(2, 2)

    assert default_block_policy("b", FooBlock())
    assert not default_block_policy("", FooBlock())
    assert not default_block_policy("l", nn.Linear(2, 2))
    frozen = FooBlock().requires_grad_(False)
    assert not default_block_policy("b", frozen)

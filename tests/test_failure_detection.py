"""Failure detection without any GPU fault: heartbeats in a TCPStore, a gloo rank that
leaves before a collective (the survivor gets an error instead of hanging), an
interrupted checkpoint write, KV-cache overflow, and a peer whose gradient is forged."""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from saint_llm_b200.utils.heartbeat import Heartbeat, HeartbeatMonitor, stale_ranks


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_heartbeat_detects_a_silent_rank():
    store = dist.TCPStore("127.0.0.1", _port(), 3, is_master=True, wait_for_workers=False)
    beats = [Heartbeat(store, r, interval=0.05).start() for r in range(3)]
    mon = HeartbeatMonitor(store, 3, timeout=0.5)
    time.sleep(0.2)
    assert mon.stale() == []
    beats[2].stop()
    time.sleep(0.8)
    assert mon.stale() == [2]
    with pytest.raises(RuntimeError, match=r"\[2\]"):
        mon.raise_if_stale()
    assert stale_ranks(store, 4, 0.5) == [2, 3]  # rank 3 never beat
    for b in beats[:2]:
        b.stop()


def _leaver(rank, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=4))
    if rank == 1:
        os._exit(0)  # leaves between steps: never joins the next collective
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))


@pytest.mark.distributed
def test_survivor_errors_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q, port = ctx.Queue(), _port()
    ps = [ctx.Process(target=_leaver, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    kind, waited = q.get(timeout=120)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert kind != "no error" and waited < 60, (kind, waited)


def test_interrupted_checkpoint_keeps_previous(tmp_path, monkeypatch):
    from saint_llm_b200.train import checkpoint as ck

    model = torch.nn.Linear(4, 4)
    path = tmp_path / "ckpt.pt"
    ck.save_checkpoint(path, model, step=1)

    def boom(obj, f, *a, **k):
        with open(f, "wb") as fh:
            fh.write(b"partial")
        raise KeyboardInterrupt

    monkeypatch.setattr(torch, "save", boom)
    with pytest.raises(KeyboardInterrupt):
        ck.save_checkpoint(path, model, step=2)
    monkeypatch.undo()
    assert ck.load_checkpoint(path, torch.nn.Linear(4, 4))["step"] == 1


def test_kv_cache_overflow_is_a_clean_error():
    from saint_llm_b200.infer.kv_cache import SWAKVCacheLayer

    c = SWAKVCacheLayer(4, 8)
    c.append(torch.zeros(1, 3, 8), torch.zeros(1, 3, 8))
    with pytest.raises(RuntimeError, match="overflow"):
        c.append(torch.zeros(1, 2, 8), torch.zeros(1, 2, 8))


def test_forged_gradient_is_rejected_and_reputation_drops():
    from saint_llm_b200.parallel import trust

    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(6, 3))
    x, y = torch.randn(5, 6), torch.randn(5, 3)
    loss_fn = lambda mod, a, b: (mod(a) - b).square().mean()  # noqa: E731
    bad, names = trust.random_peer_gradient(m, seed=4)
    nan = [torch.full_like(g, float("nan")) for g in bad]
    tr = trust.PeerReputationTracker()
    rnd = trust.DecentralizedTrainingRound(verifier=trust.GradientVerifier(m, loss_fn), tracker=tr)
    res = rnd.process([trust.PeerSubmission("rand", bad, names, x, y), trust.PeerSubmission("nan", nan, names, x, y)])
    assert res.n_accepted == 0 and tr.score("rand") < 0.5 and tr.score("nan") < 0.5

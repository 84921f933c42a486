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


def test_stale_ranks_with_a_local_store():
    """A rank that never beat, one that beat long ago and one that is fresh, judged against an
    explicit clock; the monitor raises naming the stale ranks."""
    import time

    import torch.distributed as dist

    from saint_llm_b200.utils.heartbeat import Heartbeat, HeartbeatMonitor, stale_ranks

    store = dist.HashStore()
    Heartbeat(store, 0).beat()
    store.set("hb/1", f"{time.time() - 100:.6f},3")
    now = time.time()
    assert stale_ranks(store, 3, timeout=10.0, now=now) == [1, 2]
    assert stale_ranks(store, 3, timeout=1000.0, now=now) == [2]
    store.set("hb/2", "garbage")
    assert 2 in stale_ranks(store, 3, timeout=1000.0, now=now)
    with pytest.raises(RuntimeError, match=r"ranks \[1, 2\]"):
        HeartbeatMonitor(store, 3, timeout=10.0).raise_if_stale()
    hb = Heartbeat(store, 1, interval=0.05).start()
    time.sleep(0.2)
    hb.stop()
    assert 1 not in stale_ranks(store, 2, timeout=5.0)


def test_checkpoint_rotator_keeps_the_last_n(tmp_path):
    from saint_llm_b200.train.schedule import CheckpointRotator

    class _T:
        step = 0

        def save(self, path, extra=None):
            path.write_text(str(extra))

    rot = CheckpointRotator(tmp_path / "ckpt.pt", keep_last_n=2)
    t = _T()
    for s in range(4):
        t.step = s
        rot.save(t, extra={"s": s})
    names = [p.name for p in rot.saved_paths]
    assert names == ["ckpt.step2.pt", "ckpt.step3.pt"]
    assert sorted(p.name for p in tmp_path.iterdir()) == names
    with pytest.raises(ValueError):
        CheckpointRotator(tmp_path / "x.pt", keep_last_n=0)


def test_warmup_cosine_schedule_shape_and_validation():
    from saint_llm_b200.train.schedule import warmup_cosine_schedule

    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    sched = warmup_cosine_schedule(opt, warmup_steps=4, total_steps=20, min_lr_ratio=0.1)
    lrs = []
    for _ in range(20):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        sched.step()
    assert lrs[0] < 1e-6 and abs(max(lrs) - 1.0) < 1e-6 and lrs.index(max(lrs)) == 4
    assert all(a >= b - 1e-9 for a, b in zip(lrs[4:], lrs[5:]))  # monotone decay after warm-up
    assert min(lrs[4:]) >= 0.1 - 1e-6
    for kw in ({"warmup_steps": -1, "total_steps": 5}, {"warmup_steps": 5, "total_steps": 5},
               {"warmup_steps": 1, "total_steps": 5, "min_lr_ratio": 2.0}):
        with pytest.raises(ValueError):
            warmup_cosine_schedule(opt, **kw)

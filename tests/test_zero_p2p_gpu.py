"""Hybrid ZeRO over peer memory (``csrc/zero.cu``, ``parallel.zero_p2p``) with two ranks
emulated on one GPU: every rank's announcement runs before any rank's pull, so no wait is
pending while another emulated rank still has to launch."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(64, 32), (17,), (128, 128), (5, 3), (300, 96)]
KINDS = ["muon", "adamw", "muon", "adamw", "muon"]


def _setup(cuda, ws=2):
    from saint_llm_b200.parallel.ep_p2p import EmulatedHeap
    from saint_llm_b200.parallel.zero_p2p import PeerZeroSync

    torch.manual_seed(0)
    base = [torch.randn(s, device=cuda).to(torch.bfloat16) for s in SHAPES]
    syncs, params = [], []
    for h in EmulatedHeap.create(ws, cuda):
        ps = [torch.nn.Parameter(b.clone()) for b in base]
        syncs.append(PeerZeroSync(ps, KINDS, heap=h, device=cuda, timeout_s=5.0))
        params.append(ps)
    return syncs, params


def test_peer_zero_reduce_and_broadcast(cuda):
    from saint_llm_b200.ops.gemm import check_errors

    syncs, params = _setup(cuda)
    ws = len(syncs)
    assert {syncs[0].owner[i] for i in range(len(SHAPES))} == {0, 1}, "both ranks own something"
    for step in range(2):  # the epoch advances; flags are never reset
        gs = [[torch.randn(s, device=cuda) for s in SHAPES] for _ in range(ws)]
        for r in range(ws):
            for p, g in zip(params[r], gs[r], strict=True):
                p.main_grad.copy_(g)
        for s in syncs:
            s._signal(0)
        for s in syncs:
            s._pull(s._owned_chunks_all, 0, 8)
        torch.cuda.synchronize()
        check_errors(cuda)
        for i in range(len(SHAPES)):
            o = syncs[0].owner[i]
            want = (gs[0][i] + gs[1][i]) * 0.5
            assert torch.equal(params[o][i].main_grad, want), (step, i)
        # owners update their parameters, then announce; every rank pulls what it does not own
        for r in range(ws):
            for i, p in enumerate(params[r]):
                if syncs[r].owner[i] == r:
                    p.data.add_(float(step + 1 + r))
        want_p = [params[syncs[0].owner[i]][i].detach().clone() for i in range(len(SHAPES))]
        for s in syncs:
            s.publish_params()
        for s in syncs:
            s.pull_params()
        torch.cuda.synchronize()
        check_errors(cuda)
        for r in range(ws):
            for i in range(len(SHAPES)):
                assert torch.equal(params[r][i].data, want_p[i]), (step, r, i)
    # parameters and gradients live in the arenas
    for r in range(ws):
        lo, hi = syncs[r].parena.local.data_ptr(), syncs[r].parena.local.data_ptr() + syncs[r].parena.local.numel()
        assert all(lo <= p.data_ptr() < hi for p in params[r])


def test_peer_zero_pull_times_out_cleanly(cuda):
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.parallel.ep_p2p import EmulatedHeap
    from saint_llm_b200.parallel.zero_p2p import PeerZeroSync

    ps = [torch.nn.Parameter(torch.randn(s, device=cuda).to(torch.bfloat16)) for s in SHAPES]
    s = PeerZeroSync(ps, KINDS, heap=EmulatedHeap.create(2, cuda)[0], device=cuda, timeout_s=0.2)
    s._signal(0)  # the emulated peer never announces
    s._pull(s._owned_chunks_all, 0, 4)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer timeout"):
        check_errors(cuda)
    assert float((torch.ones(3, device=cuda) * 2).sum()) == 6.0

"""Tensor-parallel peer-memory reductions (``csrc/tp.cu``, ``gemm_peer_push``) with the TP ranks
emulated on one GPU: every rank's producer runs before any rank's reduce, so no wait is ever
pending while a kernel of another emulated rank still has to run.  Compared against the fp32
sum of the ranks' products."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _comms(ws, dev, max_elems, timeout_s=5.0):
    from saint_llm_b200.parallel.ep_p2p import EmulatedHeap
    from saint_llm_b200.parallel.tp_p2p import PeerTPComm

    return [PeerTPComm(h, max_elems, timeout_s=timeout_s) for h in EmulatedHeap.create(ws, dev)]


@pytest.mark.parametrize("ws,M,N,K", [(2, 8192, 2048, 512), (2, 300, 264, 128), (4, 1000, 512, 256)])
def test_gemm_peer_push_then_reduce(cuda, ws, M, N, K):
    from saint_llm_b200.ops import gemm
    from saint_llm_b200.ops.gemm import check_errors

    comms = _comms(ws, cuda, M * N)
    torch.manual_seed(M + ws)
    for call in range(3):  # both parities, cumulative arrival counts
        xs = [torch.randn(M, K, device=cuda).to(torch.bfloat16) for _ in range(ws)]
        ws_ = [(torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16) for _ in range(ws)]
        outs = [c.produce_gemm(x, w) for c, x, w in zip(comms, xs, ws_, strict=True)]
        # the local output is exactly the plain GEMM's
        for o, x, w in zip(outs, xs, ws_, strict=True):
            assert torch.equal(o, gemm.gemm_nt(x, w))
        partial = [o.clone() for o in outs]
        for c, o in zip(comms, outs, strict=True):
            c.reduce(o)
        torch.cuda.synchronize()
        check_errors(cuda)
        want = sum(p.float() for p in partial)
        for o in outs:
            assert torch.equal(o, outs[0]), "ranks disagree"
        torch.testing.assert_close(outs[0].float(), want, rtol=1e-2, atol=1e-2)
        ref = sum(x.float() @ w.float().t() for x, w in zip(xs, ws_, strict=True))
        torch.testing.assert_close(outs[0].float(), ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("ws,n", [(2, 4096 * 256), (3, 8 * 1001)])
def test_peer_allreduce_copy(cuda, ws, n):
    from saint_llm_b200.ops.gemm import check_errors

    comms = _comms(ws, cuda, n)
    for call in range(3):
        xs = [torch.randn(n, device=cuda).to(torch.bfloat16) for _ in range(ws)]
        bufs = [c.produce_copy(x) for c, x in zip(comms, xs, strict=True)]
        for x, b in zip(xs, bufs, strict=True):
            assert b.data_ptr() != x.data_ptr() and torch.equal(b, x)
        for c, b in zip(comms, bufs, strict=True):
            c.reduce(b)
        torch.cuda.synchronize()
        check_errors(cuda)
        want = torch.zeros(n, device=cuda)
        for x in xs:
            want += x.float()
        for b in bufs:
            assert torch.equal(b, bufs[0])
        torch.testing.assert_close(bufs[0].float(), want.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)


def test_tp_reduce_times_out_cleanly(cuda):
    """A reduce whose peer never produced: the wait gives up after its limit, records the
    error, leaves x unreduced, and the context stays usable."""
    from saint_llm_b200.ops.gemm import check_errors

    comms = _comms(2, cuda, 1024, timeout_s=0.2)
    x = torch.randn(1024, device=cuda).to(torch.bfloat16)
    keep = x.clone()
    comms[0].expect[1] = 5  # arrivals that never come
    comms[0].reduce(x)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer timeout"):
        check_errors(cuda)
    assert torch.equal(x, keep)
    assert float((torch.ones(3, device=cuda) * 2).sum()) == 6.0

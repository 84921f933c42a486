"""Peer-memory expert parallelism (csrc/ep.cu) on one GPU: ``ws`` ranks are emulated in
one process, each stage run for every rank before the next stage starts, so every wait
is already satisfied when its kernel runs.  Outputs and all gradients are compared with
the fp32 eager oracle of the same routed-expert computation over the full expert set."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _bf(t):
    return t.to(torch.bfloat16).float()


def _rel(x, y):
    return ((x.float() - y.float()).norm() / (y.float().norm() + 1e-12)).item()


def _oracle(h, idx, gate, wg, wu, wd):
    out = torch.zeros_like(h)
    for e in range(wg.shape[0]):
        tok, slot = (idx == e).nonzero(as_tuple=True)
        if tok.numel():
            x = h[tok]
            y = (F.silu((x @ wg[e].t()).clamp(max=10.0)) * (x @ wu[e].t()).clamp(-10.0, 10.0)) @ wd[e].t()
            out = out.index_add(0, tok, gate[tok, slot].unsqueeze(-1) * y)
    return out


@pytest.mark.parametrize("ws,T,E,k,D,I", [(1, 300, 8, 2, 256, 128), (2, 300, 8, 2, 256, 128),
                                          (4, 257, 16, 4, 512, 384)])
def test_p2p_dispatch_combine_emulated(cuda, ws, T, E, k, D, I):
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.parallel.ep_p2p import FORWARD_STAGES, EmulatedHeap, EPCall, P2PExpertComm

    torch.manual_seed(0)
    wg, wu = (_bf(torch.randn(E, I, D, device=cuda) * 0.05) for _ in range(2))
    wd = _bf(torch.randn(E, D, I, device=cuda) * 0.05)
    hs = [_bf(torch.randn(T, D, device=cuda)) for _ in range(ws)]
    idxs = [torch.stack([torch.randperm(E, device=cuda)[:k] for _ in range(T)]) for _ in range(ws)]
    gates = [torch.rand(T, k, device=cuda) for _ in range(ws)]
    douts = [torch.randn(T, D, device=cuda) for _ in range(ws)]

    # oracle: every rank's tokens through all experts; weight grads summed over ranks
    W = [w.clone().requires_grad_(True) for w in (wg, wu, wd)]
    ref = []
    for r in range(ws):
        h = hs[r].clone().requires_grad_(True)
        g = gates[r].clone().requires_grad_(True)
        y = _oracle(h, idxs[r], g, *W)
        y.backward(douts[r])
        ref.append((y.detach(), h.grad, g.grad))

    heaps = EmulatedHeap.create(ws, cuda)
    comms = [P2PExpertComm(heaps[r], n_experts=E, hidden=D, top_k=k, timeout_s=2.0) for r in range(ws)]
    el = E // ws
    sl = [slice(r * el, (r + 1) * el) for r in range(ws)]
    bf = torch.bfloat16
    for step in range(2):  # the second step reuses every buffer with advanced epochs
        calls = [EPCall(comms[r], 7, hs[r].to(bf), idxs[r], gates[r], wg[sl[r]].to(bf), wu[sl[r]].to(bf),
                        wd[sl[r]].to(bf), (10.0, -10.0, 10.0)) for r in range(ws)]
        outs = [None] * ws
        for stage in FORWARD_STAGES:
            for r in range(ws):
                outs[r] = getattr(calls[r], stage)()
        for r in range(ws):
            calls[r].b1_push(douts[r].to(bf))
        for r in range(ws):
            calls[r].b2_experts()
        res = [calls[r].b3_pull() for r in range(ws)]
        torch.cuda.synchronize()
        check_errors(cuda)
        for r in range(ws):
            y0, dh0, dg0 = ref[r]
            dh, dgate, dwg, dwu, dwd = res[r]
            assert _rel(outs[r], y0) < 1e-2, (step, r)
            assert _rel(dh, dh0) < 2e-2, (step, r)
            assert _rel(dgate, dg0) < 2e-2, (step, r)
            assert _rel(dwg, W[0].grad[sl[r]]) < 2e-2, (step, r)
            assert _rel(dwu, W[1].grad[sl[r]]) < 2e-2, (step, r)
            assert _rel(dwd, W[2].grad[sl[r]]) < 2e-2, (step, r)


def test_p2p_wait_times_out_cleanly(cuda):
    """A flag that nothing sets: the wait gives up after its limit, records the error and the
    context stays usable."""
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.gemm import check_errors, error_word
    from saint_llm_b200.parallel.ep_p2p import PH_DX, EmulatedHeap, P2PExpertComm

    comm = P2PExpertComm(EmulatedHeap.create(2, cuda)[0], n_experts=4, hidden=64, top_k=1, timeout_s=0.2)
    comm.ensure(4)
    dh = torch.empty(4, 64, dtype=torch.bfloat16, device=cuda)
    gpos = torch.zeros(4, 1, dtype=torch.int32, device=cuda)
    backend.ext().ep_dispatch_bwd(comm.dx.ptrs, gpos, comm.C, dh, comm.flags.local.view(torch.int32), PH_DX, 2, 1,
                                  comm.timeout_ns, error_word(cuda))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer timeout"):
        check_errors(cuda)
    assert float((torch.ones(3, device=cuda) * 2).sum()) == 6.0

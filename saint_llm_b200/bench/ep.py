"""NVLink roofline of the peer-memory expert-parallel kernels (``csrc/ep.cu``).

    python -m torch.distributed.run --nproc-per-node N -m saint_llm_b200.bench.ep \
        [--tokens 8192] [--dim 2048] [--experts 64] [--topk 6] [--iters 10]

One rank per GPU.  Each phase is timed on the device with CUDA events, every rank
synchronised and at a barrier before it, and reported as the max over ranks:

* dispatch      ep_dispatch + ep_signal + ep_wait_zero (until every row has arrived)
* combine       ep_combine (pull the k rows of each token from their owners + reduce)
* combine_bwd   ep_combine_bwd + ep_signal + ep_wait_zero (push dy until arrived)
* dispatch_bwd  ep_dispatch_bwd (pull and sum the input gradients)

Roofline: the bytes that must cross NVLink per rank (rows whose owner is another rank,
``rows * dim * 2``) over the measured per-direction peer bandwidth, 770 GB/s (nominal
900); the achieved fraction is roofline time / measured time.  Routing is uniform, so
about (N-1)/N of the rows cross NVLink.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--dim", type=int, default=2048)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=6)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    rank, ws = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.gemm import check_errors, error_word
    from saint_llm_b200.ops.moe_native import RoutePlan
    from saint_llm_b200.parallel.ep_p2p import PH_CNT, PH_DX, PH_DY, PH_X, PH_Y, P2PExpertComm, SymmetricHeap

    ext = backend.ext()
    T, D, E, k = args.tokens, args.dim, args.experts, args.topk
    comm = P2PExpertComm(SymmetricHeap(None, dev), n_experts=E, hidden=D, top_k=k, timeout_s=20.0)
    comm.ensure(T)
    C = comm.C
    err = error_word(dev)
    flags = comm.flags.local.view(torch.int32)
    torch.manual_seed(rank)
    h = torch.randn(T, D, device=dev, dtype=torch.bfloat16)
    idx = torch.argsort(torch.rand(T, E, device=dev), dim=1)[:, :k].contiguous()  # k distinct experts
    gate = torch.rand(T, k, device=dev)
    dout = torch.randn(T, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty(T, D, device=dev, dtype=torch.bfloat16)
    dh = torch.empty_like(out)
    ypair = torch.empty(T * k, D, device=dev, dtype=torch.bfloat16)
    dgate = torch.empty(T, k, device=dev)
    xb = comm.xr
    x_rows, y_rows, dy_rows = comm.rows(xb), comm.rows(comm.y), comm.rows(comm.dy)

    # routing layout (untimed)
    plan = RoutePlan(idx, E, k)
    e = comm.next_epoch(PH_CNT)
    ext.ep_post_counts(plan.counts, comm.cnt.ptrs, comm.flags.ptrs, rank, e & 1, e)
    gpos = torch.empty(T, k, dtype=torch.int32, device=dev)
    el = E // ws
    ss, sr, sp = (torch.empty(el, dtype=torch.int32, device=dev) for _ in range(3))
    ext.ep_plan(idx.reshape(-1).contiguous(), plan.pos, plan.seg_start, comm.cnt.local.view(torch.int32), flags,
                e & 1, e, rank, ws, C, gpos, ss, sr, sp, comm.timeout_ns, err)
    remote_rows = int(((gpos >= 0) & (gpos // C != rank)).sum())
    y_rows.normal_()

    def dispatch() -> None:
        ext.ep_dispatch(h, gpos, C, xb.ptrs, err)
        ep = comm.next_epoch(PH_X)
        ext.ep_signal(comm.flags.ptrs, PH_X, rank, ep)
        ext.ep_wait_zero(flags, PH_X, ws, ep, x_rows, ss, sr, comm.timeout_ns, err)

    def combine() -> None:
        ep = comm.next_epoch(PH_Y)
        ext.ep_signal(comm.flags.ptrs, PH_Y, rank, ep)
        ext.ep_combine(comm.y.ptrs, gpos, gate, C, out, ypair, flags, PH_Y, ws, ep, comm.timeout_ns, err)

    def combine_bwd() -> None:
        ext.ep_combine_bwd(dout, ypair, gate, gpos, C, comm.dy.ptrs, dgate, err)
        ep = comm.next_epoch(PH_DY)
        ext.ep_signal(comm.flags.ptrs, PH_DY, rank, ep)
        ext.ep_wait_zero(flags, PH_DY, ws, ep, dy_rows, ss, sr, comm.timeout_ns, err)

    def dispatch_bwd() -> None:
        ep = comm.next_epoch(PH_DX)
        ext.ep_signal(comm.flags.ptrs, PH_DX, rank, ep)
        ext.ep_dispatch_bwd(comm.dx.ptrs, gpos, C, dh, flags, PH_DX, ws, ep, comm.timeout_ns, err)

    def timed(fn) -> float:  # noqa: ANN001
        for _ in range(args.warmup):
            torch.cuda.synchronize()
            dist.barrier()
            fn()
        ms = []
        for _ in range(args.iters):
            torch.cuda.synchronize()
            dist.barrier()
            s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            t.record()
            torch.cuda.synchronize()
            ms.append(s.elapsed_time(t))
        v = torch.tensor([sorted(ms)[len(ms) // 2]], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())

    res = {}
    link_bytes = remote_rows * D * 2
    roof_ms = link_bytes / (LINK_GBS * 1e9) * 1e3
    for name, fn in (("dispatch", dispatch), ("combine", combine), ("combine_bwd", combine_bwd),
                     ("dispatch_bwd", dispatch_bwd)):
        ms = timed(fn)
        res[name] = {"ms": round(ms, 4), "nvlink_gbs": round(link_bytes / (ms * 1e-3) / 1e9, 1),
                     "frac_of_770": round(roof_ms / ms, 3)}
    torch.cuda.synchronize()
    check_errors(dev)
    comm.close()
    if rank == 0:
        print(json.dumps({"bench": "ep_p2p", "n_gpus": ws, "tokens_per_rank": T, "dim": D, "experts": E, "topk": k,
                          "remote_rows_rank0": remote_rows, "nvlink_bytes_rank0": link_bytes,
                          "roofline_ms": round(roof_ms, 4), "phases": res}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

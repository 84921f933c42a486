"""Roofline of the tensor-parallel row-parallel projection with its all-reduce
(``gemm_peer_push`` + ``tp_reduce`` of ``csrc/tp.cu``) against the same GEMM followed by an
NCCL all-reduce.

    python -m torch.distributed.run --nproc-per-node 2 -m saint_llm_b200.bench.tp \
        [--tokens 8192] [--dim 2048] [--k 4096] [--iters 20]

One rank per GPU.  Shapes default to the attention output projection of the config-3
architecture with TP=2 (8192 tokens per micro-batch, 8 groups x 1024 split over 2 ranks, model
dim 2048).  Each variant is timed on the device with CUDA events after a device sync and a
barrier, median over iterations, max over ranks:

* fused      one GEMM whose epilogue pushes every output tile to the peers, then the reduce
* gemm_nccl  the plain tcgen05 GEMM, then ``dist.all_reduce`` of its bf16 output
* gemm       the plain GEMM alone (the compute floor)
* push       the peer all-reduce of an existing tensor (copy kernel + reduce)

Roofline: the slower of the GEMM's FLOPs at the measured bf16 peak and the bytes each rank
must send over NVLink ((ws - 1) x tokens x dim x 2) at the measured 770 GB/s per direction;
fraction = roofline time / measured time.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _peak_tflops() -> float:
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--dim", type=int, default=2048)
    ap.add_argument("--k", type=int, default=4096, help="per-rank input features of the projection")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    rank, ws = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from saint_llm_b200.ops import gemm
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.parallel.tp_p2p import PeerTPComm

    T, D, K = args.tokens, args.dim, args.k
    comm = PeerTPComm.create(None, dev, T * D, timeout_s=20.0)
    torch.manual_seed(rank)
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(D, K, device=dev) / K ** 0.5).to(torch.bfloat16)
    y = torch.randn(T, D, device=dev).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > L2

    def fused() -> None:
        comm.gemm_allreduce(x, w)

    def gemm_nccl() -> None:
        dist.all_reduce(gemm.gemm_nt(x, w))

    def gemm_only() -> None:
        gemm.gemm_nt(x, w)

    def push() -> None:
        comm.allreduce(y)

    def timed(fn) -> float:  # noqa: ANN001
        for _ in range(args.warmup):
            torch.cuda.synchronize()
            dist.barrier()
            fn()
        ms = []
        for _ in range(args.iters):
            flush.zero_()
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

    # correctness of the fused result against the NCCL one before timing
    a = comm.gemm_allreduce(x, w).clone()
    b = gemm.gemm_nt(x, w)
    dist.all_reduce(b)
    torch.cuda.synchronize()
    check_errors(dev)
    rel = ((a.float() - b.float()).norm() / b.float().norm()).item()

    flops = 2.0 * T * D * K
    link_bytes = (ws - 1) * T * D * 2
    roof_ms = max(flops / (_peak_tflops() * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3
    res = {}
    for name, fn in (("fused", fused), ("gemm_nccl", gemm_nccl), ("gemm", gemm_only), ("push", push)):
        ms = timed(fn)
        res[name] = {"ms": round(ms, 4)}
        if name != "push":
            res[name]["tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
            res[name]["frac_of_roofline"] = round(roof_ms / ms, 3)
        else:
            res[name]["nvlink_gbs"] = round(link_bytes / (ms * 1e-3) / 1e9, 1)
            res[name]["frac_of_770"] = round(link_bytes / (LINK_GBS * 1e9) * 1e3 / ms, 3)
    torch.cuda.synchronize()
    check_errors(dev)
    comm.close()
    if rank == 0:
        print(json.dumps({"bench": "tp_p2p", "n_gpus": ws, "tokens": T, "dim": D, "k_per_rank": K,
                          "fused_vs_nccl_rel": rel, "roofline_ms": round(roof_ms, 4),
                          "peak_tflops": _peak_tflops(), "l2": "256 MB written between iterations",
                          "variants": res}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

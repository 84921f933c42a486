"""Worker for the multi-GPU expert-parallel test (launched by torch.distributed.run, one
rank per GPU): the same MoE layer with all experts local vs sharded over the ranks with
the peer-memory transport and with the NCCL transport.  Rank 0 prints one JSON line."""

import copy
import datetime
import faulthandler
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _rel(x, y):
    return ((x.float() - y.float()).norm() / (y.float().norm() + 1e-12)).item()


def main() -> None:
    faulthandler.enable()
    rank, ws = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from saint_llm_b200.config import MoEConfig
    from saint_llm_b200.models.moe import DeepSeekMoE
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.parallel import ep

    cfg = MoEConfig(hash_routed_layers=0, shared_experts=1, routed_experts=8, experts_per_token=2,
                    expert_intermediate_dim=256)
    torch.manual_seed(0)
    full = DeepSeekMoE(512, cfg, layer_idx=3, use_grouped_gemm=True).to(dev).to(torch.bfloat16)
    copies = {t: copy.deepcopy(full) for t in ("p2p", "nccl")}  # before any forward (non-leaf attributes)
    torch.manual_seed(1 + rank)
    x = torch.randn(2, 192, 512, device=dev, dtype=torch.bfloat16)
    g = torch.randn_like(x)
    res = {}
    xr = x.clone().requires_grad_(True)
    y_ref = full(xr)
    y_ref.backward(g)
    w_ref = [p.grad.clone() for p in (full.grouped_experts.gate_weight, full.grouped_experts.up_weight,
                                      full.grouped_experts.down_weight)]
    for w in w_ref:
        dist.all_reduce(w)
    el = cfg.routed_experts // ws
    for transport in ("p2p", "nccl"):
        m = copies[transport]
        m.zero_grad()
        ep.shard_grouped_experts(m, rank, ws, None)
        if transport == "p2p":
            from saint_llm_b200.parallel.ep_p2p import attach_p2p_comm

            attach_p2p_comm(m, None, dev, timeout_s=20.0)
        for it in range(2):
            m.zero_grad()
            xe = x.clone().requires_grad_(True)
            y = m(xe)
            y.backward(g)
        torch.cuda.synchronize()
        check_errors(dev)
        if transport == "p2p":
            m.ep_comm.close()  # collective; no rank frees memory a peer may still read
        ge = m.grouped_experts
        res[transport] = {
            "out": _rel(y, y_ref), "dx": _rel(xe.grad, xr.grad),
            "dw": max(_rel(p.grad, w[rank * el:(rank + 1) * el]) for p, w in
                      zip((ge.gate_weight, ge.up_weight, ge.down_weight), w_ref, strict=True)),
        }
    worst = {t: max(v.values()) for t, v in res.items()}
    t = torch.tensor([worst["p2p"], worst["nccl"]], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({"ws": ws, "p2p_max_rel": t[0].item(), "nccl_max_rel": t[1].item()}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Worker for the multi-GPU tensor-parallel test (launched by torch.distributed.run, one rank
per GPU): a 2-layer bf16 model with attention heads sharded over the ranks, once with the
NVLink peer-memory transport and once with NCCL, against the unsharded model.  Rank 0 prints
one JSON line."""

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
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.parallel.tp import apply_tensor_parallel

    cfg = ModelConfig.bench_tiny().model_copy(update={"n_layers": 2})
    torch.manual_seed(0)
    full = SaintLLM(cfg).to(dev).to(torch.bfloat16)
    models = {"p2p": copy.deepcopy(full), "nccl": copy.deepcopy(full)}
    B, T = 2, 256
    torch.manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (B, T), device=dev)
    res = {}
    out_full = full(ids)["logits"]
    syncs = {t: apply_tensor_parallel(m, None, transport=t, max_tokens=B * T) for t, m in models.items()}
    logits, grads = {}, {}
    for t, m in models.items():
        for it in range(2):  # the second pass reuses the receive parities and counters
            m.zero_grad(set_to_none=True)
            out = m(ids)["logits"]
            loss = out.float().logsumexp(-1).mean()
            loss.backward()
            syncs[t]()
        torch.cuda.synchronize()
        check_errors(dev)
        logits[t] = out.detach()
        grads[t] = {n: p.grad.detach().float() for n, p in m.named_parameters() if p.grad is not None}
    res["p2p_vs_nccl_logits"] = _rel(logits["p2p"], logits["nccl"])
    res["p2p_vs_full_logits"] = _rel(logits["p2p"], out_full.detach())
    worst = 0.0
    for n, g in grads["nccl"].items():
        if g.norm() > 0:
            worst = max(worst, _rel(grads["p2p"][n], g))
    res["p2p_vs_nccl_grad_max_rel"] = worst
    res["n_grads"] = len(grads["nccl"])
    gathered = [torch.empty_like(logits["p2p"]) for _ in range(ws)]
    dist.all_gather(gathered, logits["p2p"].contiguous())
    res["ranks_identical"] = all(torch.equal(g, gathered[0]) for g in gathered)
    syncs["p2p"].comm.close()
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

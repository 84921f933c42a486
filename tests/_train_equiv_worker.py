"""Worker for the multi-GPU training-step equivalence test.

``--mode single``: one process trains the reduced config-3 model (2 layers) on the whole
global token set (G sequences, one micro-batch per sequence, gradient accumulation) for S
steps.  ``--mode ep`` (under torch.distributed.run, one rank per GPU): the same model and
seed with the experts sharded over the ranks (EP = world size), hybrid ZeRO for the
replicated weights (NCCL or peer-memory transport, optionally reduced from the blocks'
backward hooks) and the chosen token transport; rank r trains on sequences
[r*G/N, (r+1)*G/N) with the same micro-batch size.  The same global batch is used every
step, so the loss falls visibly and a wrong update shows.  Each run writes its per-step
global-mean losses as JSON to ``--out``."""

import argparse
import datetime
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def build(dev, world, transport, zero, zero_transport="nccl", overlap=False):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.train.engine import attach_main_grads, cast_params

    cfg = ModelConfig.bench_16b().model_copy(update={"n_layers": 2, "linear_quant": "bf16"})
    torch.manual_seed(0)
    with torch.device(dev):
        model = SaintLLM(cfg)
    cast_params(model, torch.bfloat16)
    sync = None
    if world > 1:
        from saint_llm_b200.parallel import ep

        sync = ep.setup_expert_parallel(model, transport=transport, zero=zero, zero_transport=zero_transport,
                                        overlap_reduce=overlap)
    params = attach_main_grads(model)
    muon, adamw = split_for_muon_adamw(model)
    opt = MuonAdamW(muon, adamw, lr=2.7e-4, qk_clip_layers=model.attention_layers())
    if sync is not None:
        sync.configure_optimizer(opt)
    return cfg, model, opt, params, sync


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["single", "ep"], required=True)
    ap.add_argument("--transport", default="p2p")
    ap.add_argument("--no-zero", action="store_true")
    ap.add_argument("--zero-transport", default="nccl", choices=["nccl", "p2p"])
    ap.add_argument("--overlap", action="store_true", help="reduce gradients from the blocks' backward hooks")
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    if a.mode == "ep":
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.step import TrainStep

    cfg, model, opt, params, sync = build(dev, world, a.transport, not a.no_zero, a.zero_transport, a.overlap)
    g = torch.Generator().manual_seed(1234)
    tokens = torch.randint(0, cfg.vocab_size, (a.seqs, 1, a.seq_len), generator=g)
    per = a.seqs // world
    mine = tokens[rank * per:(rank + 1) * per].to(dev)
    step = TrainStep(model, opt, micro_batches=per, params=params, grad_sync=sync)
    losses = []
    for _ in range(a.steps):
        loss = step.run_device(mine).detach().reshape(1)
        if world > 1:
            torch.distributed.all_reduce(loss)
            loss /= world
        losses.append(float(loss.item()))
    torch.cuda.synchronize()
    check_errors(dev)
    if rank == 0:
        with open(a.out, "w") as f:
            json.dump({"mode": a.mode, "world": world, "transport": a.transport, "losses": losses}, f)
    if world > 1:
        comm = getattr(model, "ep_comm", None)
        if comm is not None:
            comm.close()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

"""``bench.py --impl reference``: the unmodified reference (iZonex/saint-llm) on the same
model configuration, token count and timing rules as the framework arm.

Only the reference's public API is used: ``saint_llm_core.ModelConfig`` /
``SaintLLM``, ``saint_llm_training.make_loss_fn``, ``saint_llm_optim.split_for_muon_adamw``
+ ``Muon`` with ``torch.optim.AdamW`` (the reference's intended hyper-parameters), and for
N > 1 the reference's ``fsdp2_wrap`` (its only multi-GPU training path; it has no expert
parallelism wired into the model).  Settings the reference needs to run this model on a
B200 at all, each a public switch of the reference:
``activation_checkpointing=True`` (its attention materialises (T x T) scores), and the
per-expert module layout (``moe_use_grouped_gemm=False``; its Muon raises on the stacked
3-D expert weights).  Weights stay fp32 under bf16 autocast -- the reference's own
mixed-precision mode (``Trainer(mixed_precision="bf16")``); casting its parameters to bf16
breaks its einsums.  fp32 weights + gradients + Muon momentum of the ~16B-parameter
model need ~192 GB, more than one B200 holds, so at one GPU the arm reports
``unavailable`` with that arithmetic instead of running out of memory.

Every step accumulates gradients over the same ``seqs_per_gpu`` sequences of 4096
tokens as the framework arm, then steps the optimizers.  Timing: CUDA events around K
steps after W warm-up steps, barrier + synchronize on both sides, max over ranks.
"""

from __future__ import annotations

import datetime
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def _reference_config(ModelConfig, args):  # noqa: N803
    """Config 3 expressed with the reference's own config classes (same pinned fields)."""
    from saint_llm_core.config import AttentionConfig, MoEConfig, MTPConfig, TokenizerSlots

    n_layers = args.layers or 28
    return ModelConfig(
        n_layers=n_layers, hidden_dim=2048, vocab_size=32768, first_dense_swa_layers=0,
        attention=AttentionConfig(query_heads=16, head_dim=128),
        moe=MoEConfig(hash_routed_layers=0, shared_experts=2, routed_experts=64, experts_per_token=6,
                      expert_intermediate_dim=1408),
        mtp=MTPConfig(depth=1),
        tokenizer_slots=TokenizerSlots(image_pad=32700, audio_start=32701, audio_end=32705, video_start=32706,
                                       video_end=32707, think_start=32708, think_end=32709,
                                       memory_block_base=32710),
        linear_quant=args.linear_quant, fp8_use_real_gemm=args.linear_quant == "fp8",
        moe_use_grouped_gemm=False, activation_checkpointing=True,
    )


def run(args) -> dict:
    try:
        return _run(args)
    except Exception as e:  # noqa: BLE001 - report any failure of the reference as unavailable
        msg = f"{type(e).__name__}: {e}".splitlines()[0][:300]
        return _unavailable(f"reference run failed: {msg}")


def _run(args) -> dict:
    if not os.path.isdir(os.path.join(REF, "saint_llm_core")):
        return _unavailable("reference not installed in baseline/_ref (run baseline/install_reference.sh)")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from saint_llm_core.config import ModelConfig
    from saint_llm_core.model import SaintLLM
    from saint_llm_optim import Muon, split_for_muon_adamw
    from saint_llm_training.losses import make_loss_fn

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800), device_id=dev)
    cfg = _reference_config(ModelConfig, args)
    # parameter count from the architecture (no allocation) and the fp32 training-state footprint
    with torch.device("meta"):
        n_params = sum(p.numel() for p in SaintLLM(cfg).parameters())
    need = n_params * 12 / world  # fp32 weights + grads + Muon momentum (AdamW share is small)
    have = torch.cuda.get_device_properties(dev).total_memory
    if need > 0.95 * have:
        return _unavailable(f"reference keeps fp32 weights, grads and Muon momentum: {n_params / 1e9:.1f}B params x "
                            f"12 B / {world} GPU(s) = {need / 1e9:.0f} GB > {have / 1e9:.0f} GB per GPU")
    torch.manual_seed(0)
    with torch.device(dev):
        model = SaintLLM(cfg)
    if world > 1:
        from saint_llm_distributed.fsdp import fsdp2_wrap

        model = fsdp2_wrap(model)
    muon_params, adamw_params = split_for_muon_adamw(model)
    muon = Muon(muon_params, lr=2.7e-4)
    adamw = torch.optim.AdamW(adamw_params, lr=2.7e-4, betas=(0.9, 0.95), eps=1e-20, weight_decay=0.1)
    loss_fn = make_loss_fn(cfg.mtp, moe_cfg=cfg.moe)
    n_micro = args.seqs_per_gpu // args.micro_batch
    g = torch.Generator().manual_seed(rank)
    host = torch.randint(0, cfg.vocab_size, (n_micro, args.micro_batch, args.seq_len), generator=g).pin_memory()

    def step() -> torch.Tensor:
        total = torch.zeros((), device=dev)
        toks = host.to(dev, non_blocking=True)
        for i in range(n_micro):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = loss_fn(model, toks[i]).float() / n_micro
            loss.backward()
            total += loss.detach()
        muon.step()
        adamw.step()
        muon.zero_grad(set_to_none=True)
        adamw.zero_grad(set_to_none=True)
        return total

    budget = float(os.environ.get("SV4_REF_BUDGET_S", "1200"))
    t0 = time.perf_counter()
    for _ in range(args.warmup):
        step()
        torch.cuda.synchronize()
        if time.perf_counter() - t0 > budget:
            return _unavailable(f"reference step exceeds the time budget: {args.warmup} warm-up steps of "
                                f"{n_micro} x {args.seq_len} tokens took > {budget:.0f} s")
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        loss = step()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t = torch.tensor([start.elapsed_time(end) / args.steps], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    tokens = world * args.seqs_per_gpu * args.seq_len
    res = {
        "impl": "reference", "metric": "train tokens/sec/box (max over ranks) FP8 MoE at 1/2/4/8 B200; decode tok/s",
        "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if args.linear_quant == "bf16" else "fp8",
        "data": "synthetic uniform-random tokens; random-init weights N(0,0.02)",
        "config": {"model": "reference SaintLLM, BASELINE config 3 architecture", "n_layers": cfg.n_layers,
                   "global_batch": world * args.seqs_per_gpu, "seq_len": args.seq_len,
                   "parallelism": f"fsdp2 dp{world}" if world > 1 else "single-gpu",
                   "reference_settings": "fp32 params + bf16 autocast, activation checkpointing, "
                                         "per-expert modules",
                   "final_loss": float(loss.item())},
    }
    if world > 1:
        torch.distributed.destroy_process_group()
    return res if rank == 0 else {}

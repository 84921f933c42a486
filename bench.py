"""Headline benchmark: training tokens/s of the ~16B FP8-class MoE.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (``torchrun`` for N > 1, expert parallel EP = N, data parallel for
the replicated weights).  Per GPU a step is one optimizer step over ``seqs_per_gpu`` x
4096 uniform-random tokens (weak scaling: 32 sequences per GPU, i.e. global batch
256 x 4096 at N = 8), in micro-batches of 2 sequences on one GPU and 4 with N > 1.  The W
warm-up steps are untimed; exactly K steps are timed with
CUDA events between a barrier + synchronize on both sides; the per-rank time is
max-reduced over ranks.  Every step copies its token batch from pinned host memory
inside the timed region.  The model weights (tens of GB) stream through HBM every step,
far beyond the 126 MB L2, so no explicit L2 flush is used.

``e2e`` repeats the measurement through the public ``TrainStep`` call (host batch in,
Python float loss out) timed by the host clock around the whole call.

After the timed regions: one step with per-phase CUDA events and one under the torch
profiler (kernel counts, device-busy time, top kernels); at N = 1 with the bf16 headline a
short measurement of the block-scaled FP8 recipe (``fp8_variant``); and the decode
measurement of config 5 (``decode``: one replica per GPU, 64 prompts of 4096 tokens, 512
greedy steps).

The headline dtype is bf16 (at least the reference's precision): on this implementation the
bf16 step is faster than the FP8 recipe, whose number is reported next to it.

``--tp T`` (N divisible by T) adds config 3's tensor parallelism on attention: the T ranks
of a TP group share a batch of T x micro-batch sequences (heads split over the group, each
rank routing its micro-batch share through the MoE layers), so the tokens per GPU are
unchanged; EP stays over all N ranks and ZeRO over the N / T replicas.  Not the default:
this layout has only run on CPU ranks so far.

Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

# fewer fragmentation stalls near the 180 GB ceiling (must be set before CUDA initialises)
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

METRIC = "train tokens/sec/box (max over ranks) FP8 MoE at 1/2/4/8 B200; decode tok/s"
MODEL_DESC = ("V4-MoE ~16B total / ~2.7B active (BASELINE config 3): d2048 L28 H16x128, 64 routed top-6 + "
              "2 shared, I1408, MTP1, vocab 32768")


def _dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9], strict=True):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def count_native_launches(fn) -> tuple[int, float, list]:
    """Kernels of this framework (namespace sv4) launched by one call of fn, the summed
    device time of every kernel of that call in ms (compared with the step time it shows how
    much of the step the GPU spends between kernels), and the 15 kernels with the largest
    total time (name, launches, ms)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    kernels = [ev for ev in prof.events() if ev.device_type == torch.autograd.DeviceType.CUDA
               and "Memcpy" not in ev.name and "Memset" not in ev.name]
    busy_us = sum(ev.time_range.elapsed_us() for ev in kernels)
    per: dict[str, list[float]] = {}
    for ev in kernels:
        key = ev.name.split("(")[0][:80]
        rec = per.setdefault(key, [0, 0.0])
        rec[0] += 1
        rec[1] += ev.time_range.elapsed_us()
    top = sorted(per.items(), key=lambda kv: -kv[1][1])[:15]
    return (sum(1 for ev in kernels if "sv4::" in ev.name), busy_us / 1000.0,
            [[k, v[0], round(v[1] / 1000.0, 2)] for k, v in top])


def run_config(args, world: int):
    """The run layout of this bench as a ``RunConfig`` (consumed by ``build_training``)."""
    from saint_llm_b200.config import RunConfig

    tp = getattr(args, "tp", 1)
    # with TP the ranks of one TP group share a batch of tp x micro_batch sequences: each routes
    # micro_batch of them through the MoE layers, so the work per GPU matches tp = 1
    return RunConfig(ep=world, tp=tp, zero="dp" if args.no_zero else "hybrid_zero",
                     fused_ep=args.ep_transport == "p2p", fused_tp=getattr(args, "tp_transport", "nccl") == "p2p",
                     fused_zero=not args.no_overlap_reduce, zero_transport=args.zero_transport,
                     cuda_graphs=not args.no_cuda_graph,
                     fp8_expert_cache=args.fp8_expert_cache,
                     micro_batch=args.micro_batch * tp, seq_len=args.seq_len,
                     grad_accum=args.seqs_per_gpu // args.micro_batch, lr=2.7e-4, adamw_lr=2.7e-4,
                     pg_timeout_s=600.0, seed=0)


def build_ours(args, device, world):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.train.launch import build_training

    upd = {"linear_quant": args.linear_quant, "activation_checkpointing": args.ckpt}
    if args.layers:
        upd["n_layers"] = args.layers
    cfg = ModelConfig.bench_16b().model_copy(update=upd)
    run = run_config(args, world)
    job = build_training(cfg, run, device)
    return cfg, job.model, job.step, job


def _uniform_loss(cfg) -> float:
    """The training loss of a model that predicts every token uniformly: ln V for the main
    head plus the MTP heads' weighted ln V (the balance term is excluded)."""
    import math

    from saint_llm_b200.train.losses import mtp_weight

    w = 1.0 + sum(mtp_weight(cfg.mtp, k) for k in range(cfg.mtp.depth))
    return w * math.log(cfg.vocab_size)


def _rank_mean(x: torch.Tensor, world: int) -> float:
    t = x.detach().float().reshape(1).clone()
    if world > 1:
        torch.distributed.all_reduce(t)
        t /= world
    return float(t.item())


def run_ours(args) -> dict:
    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from saint_llm_b200.train.launch import init_distributed

        init_distributed(run_config(args, world), device)
    cfg, model, step, job = build_ours(args, device, world)
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.engine import SyntheticTokens
    from saint_llm_b200.utils.profiling import PhaseRecorder

    n_micro = args.seqs_per_gpu // args.micro_batch
    # the ranks of one TP group read the same batch (job.replica == rank without TP)
    data = SyntheticTokens(cfg.vocab_size, args.micro_batch * args.tp, args.seq_len, n_micro, seed=job.replica,
                           n_batches=args.data_pool)
    it = iter(range(1 << 30))

    def device_step():
        return step.run_device(data.batch(next(it)).to(device, non_blocking=True))

    first_loss = None
    for _ in range(args.warmup):
        loss = device_step()
        if first_loss is None:
            first_loss = _rank_mean(loss, world)
    torch.cuda.synchronize()
    check_errors(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clk:
        start.record()
        marks[0].record()
        for i in range(args.steps):
            loss = device_step()
            marks[i + 1].record()  # per-step spread (no sync: steps still queue back to back)
        end.record()
        torch.cuda.synchronize()
        per_step = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
        if world > 1:
            torch.distributed.barrier()
        t_ms = torch.tensor([start.elapsed_time(end) / args.steps], device=device)
        if world > 1:
            torch.distributed.all_reduce(t_ms, op=torch.distributed.ReduceOp.MAX)
        ms = float(t_ms.item())
        final_loss = _rank_mean(loss, world)
        check_errors(device)

    # end-to-end through the public call: host batch in, float loss out, timed on the host
    # around the calls; its own clock record (the power-capped SM clock differs between the
    # two loops by a few percent, which is what separates the two numbers)
    with ClockSampler(local) as clk_e:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(data.batch(next(it)))
        torch.cuda.synchronize()
        t_e = torch.tensor([(time.perf_counter() - t0) * 1000 / args.steps], device=device)
    if world > 1:
        torch.distributed.all_reduce(t_e, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(t_e.item())

    # one more step with per-phase CUDA events (outside the timed regions), max over ranks
    if world > 1:
        torch.distributed.barrier()
    comm = getattr(model, "ep_comm", None)
    rows0 = getattr(comm, "rows_received", 0)
    with PhaseRecorder(device) as rec:
        device_step()
    phases = rec.summary()
    expert_rows = None
    if comm is not None and world > 1:
        # expert rows (128-padded) each rank owned in that step: the load spread the EP waits absorb
        mine = torch.tensor([comm.rows_received - rows0], dtype=torch.int64, device=device)
        allr = [torch.zeros_like(mine) for _ in range(world)]
        torch.distributed.all_gather(allr, mine)
        expert_rows = [int(x.item()) for x in allr]
    n_native, busy_ms, top_kernels = count_native_launches(device_step)
    launches = n_native * args.steps
    tokens_per_step = world * args.seqs_per_gpu * args.seq_len
    result = {
        "metric": METRIC, "value": tokens_per_step / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if args.linear_quant == "bf16" else "fp8",
        "data": "synthetic uniform-random tokens; random-init weights N(0,0.02)",
        "config": {"model": MODEL_DESC, "n_layers": cfg.n_layers, "global_batch": world * args.seqs_per_gpu,
                   "seq_len": args.seq_len, "micro_batch": args.micro_batch,
                   "parallelism": (f"ep{world}" + (f"+tp{args.tp}" if args.tp > 1 else "")
                                   + f"+dp{world // args.tp}" + ("" if args.no_zero else "+zero")) if world > 1
                   else "single-gpu",
                   "tp_transport": args.tp_transport if args.tp > 1 else None,
                   "ep_transport": args.ep_transport if world > 1 else None,
                   "zero_transport": args.zero_transport if world > 1 and not args.no_zero else None,
                   "cuda_graph": bool(getattr(step, "_graph", None) is not None),
                   "cuda_graph_error": getattr(step, "graph_error", None),
                   "linear_quant": args.linear_quant, "activation_checkpointing": args.ckpt,
                   "fp8_expert_cache": args.fp8_expert_cache if args.linear_quant == "fp8" else None,
                   "l2": "inputs larger than L2 (the weights stream through HBM every step)",
                   "data_pool_batches": args.data_pool,
                   "loss": {"first_warmup": first_loss, "final": final_loss, "uniform_prediction": _uniform_loss(cfg),
                            "note": "mean over ranks; main CE + MTP-weighted CE + balance term"},
                   "final_loss": final_loss,
                   "phases_ms": phases,
                   "expert_rows_per_rank": expert_rows,
                   "step_ms_min_max_this_rank": [round(min(per_step), 1), round(max(per_step), 1)],
                   "kernel_busy_ms_per_step": round(busy_ms, 1),
                   "top_kernels_ms_per_step": top_kernels,
                   "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1)},
        "clocks": clk.summary(),
        "e2e": {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": int(data.bytes_per_step), "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms, "clocks": clk_e.summary(),
                "timing": "host perf_counter around TrainStep.__call__ (pinned host batch -> device, loss -> "
                          "host float), after a device sync and barrier; max over ranks"},
        "gpu_launches": launches,
    }
    if world > 1:
        comm = getattr(model, "ep_comm", None)
        if comm is not None:
            comm.close()  # collective: peers stop touching each other's buffers first
        tp_comm = getattr(job.grad_sync, "tp_comm", None)
        if tp_comm is not None:
            tp_comm.close()
    import gc

    del step, model
    gc.collect()
    torch.cuda.empty_cache()
    if world == 1 and args.linear_quant == "bf16" and not args.no_fp8_variant:
        result["fp8_variant"] = run_fp8_variant(args, device)
        gc.collect()
        torch.cuda.empty_cache()
    if not args.no_decode:
        result["decode"] = run_decode(args, device, world)
    if world > 1:
        torch.distributed.destroy_process_group()
    return result if rank == 0 else {}


def run_fp8_variant(args, device) -> dict:
    """The same single-GPU training step with the block-scaled FP8 recipe (config 3's
    precision): every linear the reference routes through its quantisation factory and the
    routed experts run their forward GEMMs in FP8 (bf16 straight-through backward).  Timed
    the same way as the headline (CUDA events, W warm-up steps) over min(K, 3) steps."""
    torch.cuda.reset_peak_memory_stats(device)
    fargs = argparse.Namespace(**vars(args))
    fargs.linear_quant = "fp8"
    fargs.tp = 1
    cfg, model, step, _ = build_ours(fargs, device, 1)
    from saint_llm_b200.train.engine import SyntheticTokens

    n_micro = args.seqs_per_gpu // args.micro_batch
    data = SyntheticTokens(cfg.vocab_size, args.micro_batch, args.seq_len, n_micro, seed=0, n_batches=2)
    it = iter(range(1 << 30))
    k = max(1, min(args.steps, 3))
    for _ in range(args.warmup):
        step.run_device(data.batch(next(it)).to(device, non_blocking=True))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(k):
        loss = step.run_device(data.batch(next(it)).to(device, non_blocking=True))
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / k
    out = {"value": args.seqs_per_gpu * args.seq_len / (ms / 1000.0), "unit": "tokens/s", "ms_per_step": ms,
           "steps": k, "warmup": args.warmup, "dtype": "fp8",
           "recipe": "block-scaled FP8 forward (1x128 activations, 128x128 weights) for the attention projections, "
                     "shared and routed experts; bf16 straight-through backward",
           "fp8_expert_cache": args.fp8_expert_cache, "cuda_graph": step._graph is not None,
           "final_loss": float(loss.item()),
           "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1)}
    del step, model
    return out


def run_decode(args, device, world: int) -> dict:
    """Config 5's serving measurement on every rank (one independent replica per GPU, the
    reference's only multi-GPU inference layout): 64 prompts of 4096 tokens prefilled in
    chunks, then greedy decode; box tokens/s from the slowest rank's time."""
    from saint_llm_b200.bench.decode import measure_decode

    r = measure_decode(batch=args.decode_batch, prompt=args.seq_len, steps=args.decode_steps, layers=args.layers,
                       device=device)
    B, P, S = args.decode_batch, args.seq_len, args.decode_steps
    t = torch.tensor([B * S / r["value"], B * P / r["prefill_tokens_per_s"]], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    dec_s, pre_s = float(t[0]), float(t[1])
    return {"metric": "decode tok/s", "value": world * B * S / dec_s, "unit": "tokens/s",
            "prefill_tokens_per_s": world * B * P / pre_s, "decode_ms_per_step": dec_s * 1000.0 / S,
            "n_gpus": world, "parallelism": f"{world} replica(s), one per GPU", "dtype": r["dtype"],
            "timing": "CUDA events, max over ranks; prefill and decode timed separately",
            "config": r["config"]}


def run_reference(args) -> dict:
    from baseline import reference_arm

    return reference_arm.run(args)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seqs-per-gpu", type=int, default=32)
    ap.add_argument("--micro-batch", type=int, default=None,
                    help="sequences per micro-batch (default: 2 on one GPU, where the CUDA-graph pool must fit "
                         "next to the unsharded expert pool; 4 with N > 1, where expert parallelism frees the "
                         "memory and halves the per-micro-batch gradient read-modify-writes and EP calls; the "
                         "reference arm uses 2)")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel token transport for N > 1 (peer-memory kernels or NCCL all-to-all)")
    ap.add_argument("--no-zero", action="store_true",
                    help="N > 1: all-reduce replicated gradients and update them on every rank (no hybrid ZeRO)")
    ap.add_argument("--fp8-expert-cache", default="auto", choices=["auto", "always", "never"],
                    help="FP8: keep the routed experts' FP8 weight copies between steps (auto: when sharded by EP)")
    ap.add_argument("--no-cuda-graph", action="store_true",
                    help="N = 1: launch every kernel eagerly instead of replaying the captured micro-batch graph")
    ap.add_argument("--zero-transport", default="p2p", choices=["nccl", "p2p"],
                    help="N > 1 with hybrid ZeRO: the peer-memory pull kernels (default) or NCCL reduce/broadcast")
    ap.add_argument("--no-overlap-reduce", action="store_true",
                    help="N > 1 with hybrid ZeRO: reduce gradients after the backward instead of from block hooks")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor parallelism on attention (config 3 names TP=2), composed with EP over all ranks")
    ap.add_argument("--tp-transport", default="nccl", choices=["nccl", "p2p"],
                    help="TP reductions: NCCL all-reduce, or the peer-memory fused GEMM + reduce kernels")
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--no-decode", action="store_true", help="skip the decode (config 5) measurement")
    ap.add_argument("--no-fp8-variant", action="store_true",
                    help="N = 1, bf16 headline: skip the extra FP8-recipe measurement")
    ap.add_argument("--decode-batch", type=int, default=64)
    ap.add_argument("--decode-steps", type=int, default=512)
    ap.add_argument("--data-pool", type=int, default=8,
                    help="distinct synthetic step batches cycled through (pinned host memory)")
    ap.add_argument("--linear-quant", default="bf16", choices=["bf16", "fp8"])
    ap.add_argument("--ckpt", action="store_true", help="activation checkpointing per block")
    ap.add_argument("--layers", type=int, default=0, help="(development only) override n_layers")
    args = ap.parse_args()
    if args.micro_batch is None:
        world = int(os.environ.get("WORLD_SIZE", args.gpus))
        args.micro_batch = 2 if args.impl == "reference" or world == 1 else 4
    res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

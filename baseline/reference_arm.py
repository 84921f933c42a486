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
breaks its einsums.

Every step accumulates gradients over the same ``seqs_per_gpu`` sequences of 4096
tokens as the framework arm, then steps the optimizers.  Timing: CUDA events around K
steps after W warm-up steps, barrier + synchronize on both sides, max over ranks.

Time budget (``SV4_REF_BUDGET_S``, default 600 s of wall clock from the start of the arm):
the arm first times single micro-batches (one untimed, one timed with CUDA events, max over
ranks) and one optimizer step, extrapolates the W + K steps and runs them only if they fit
the budget.  Otherwise -- and when the model's fp32 training state does not fit the GPUs at
all, in which case the micro-batches are timed on the largest layer cut that fits and scaled
linearly to the full depth -- it prints its ``unavailable`` line carrying those measured
times and the extrapolated step time, so the record shows that the reference ran on the box.

Watchdog (N > 1, ``SV4_REF_WATCHDOG_S``, default 720 s): if the probe itself has not finished by
then, rank 0 prints an ``unavailable`` line naming the stage it reached and every rank exits,
so the driver records a line instead of killing a silent arm at its own limit.  NVLink
multicast (NVLS) is off in the arm's NCCL group, so an exit leaves no peer memory bound.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
METRIC = "train tokens/sec/box (max over ranks) FP8 MoE at 1/2/4/8 B200; decode tok/s"


def _unavailable(why: str, measured: dict | None = None) -> dict:
    out: dict = {"impl": "reference", "unavailable": why}
    if measured:
        out["measured"] = measured
    return out


def _reference_config(ModelConfig, args, n_layers: int | None = None):  # noqa: N803
    """Config 3 expressed with the reference's own config classes (same pinned fields)."""
    from saint_llm_core.config import AttentionConfig, MoEConfig, MTPConfig, TokenizerSlots

    return ModelConfig(
        n_layers=n_layers or args.layers or 28, hidden_dim=2048, vocab_size=32768, first_dense_swa_layers=0,
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
        res = _run(args)
    except Exception as e:  # noqa: BLE001 - report any failure of the reference as unavailable
        msg = f"{type(e).__name__}: {e}".splitlines()[0][:300]
        res = _unavailable(f"reference run failed: {msg}")
    if res and not getattr(args, "no_decode", False) and int(os.environ.get("WORLD_SIZE", 1)) == 1:
        try:
            res["decode"] = _decode(args)
        except Exception as e:  # noqa: BLE001
            res["decode"] = {"unavailable": f"reference decode failed: {type(e).__name__}: {e}".splitlines()[0][:300]}
    return res


def _decode(args) -> dict:
    """Config 5 on one GPU through the reference's public ``greedy_decode_cached`` with its
    ``KVCacheBundle``: prefill (one forward over the prompt, as the API does) and greedy
    steps, timed as two calls (1 new token, then 1 + n new tokens; the difference is n
    decode steps).  Its prefill materialises (B, H, T, T) attention scores, so the batch is
    halved from the configured 64 until it fits; n is capped to fit the time budget and the
    step time is extrapolated to the configured step count.  Reported as measured, with
    ``unavailable`` whenever the configured batch or step count could not be run as is."""
    import gc

    from saint_llm_core.config import ModelConfig
    from saint_llm_core.model import SaintLLM
    from saint_llm_inference.generate import greedy_decode_cached

    gc.collect()
    torch.cuda.empty_cache()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    cfg = _reference_config(ModelConfig, args).model_copy(update={"activation_checkpointing": False})
    torch.manual_seed(0)
    with torch.device(dev):
        model = SaintLLM(cfg)
    model.eval()
    want_b, P, S = args.decode_batch, args.seq_len, args.decode_steps
    budget = float(os.environ.get("SV4_REF_DECODE_BUDGET_S", "240"))
    b, err = want_b, None
    while b >= 1:
        ids = torch.randint(0, cfg.vocab_size, (b, P), device=dev)
        try:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
                torch.cuda.synchronize(dev)
                ev[0].record()
                greedy_decode_cached(model, ids, max_new_tokens=1)
                ev[1].record()
                torch.cuda.synchronize(dev)
                prefill_s = ev[0].elapsed_time(ev[1]) / 1000.0
                n = 8
                ev[2].record()
                greedy_decode_cached(model, ids, max_new_tokens=1 + n)
                ev[3].record()
                torch.cuda.synchronize(dev)
                step_s = max(ev[2].elapsed_time(ev[3]) / 1000.0 - prefill_s, 1e-6) / n
            break
        except torch.OutOfMemoryError as e:
            err = str(e).splitlines()[0][:120]
            ids = None
            gc.collect()
            torch.cuda.empty_cache()
            b //= 2
    if b < 1:
        return {"unavailable": f"reference decode ran out of memory at every batch ({err})"}
    measured = {"batch_run": b, "batch_config": want_b, "prompt": P, "prefill_s": round(prefill_s, 3),
                "prefill_tokens_per_s": round(b * P / prefill_s, 1), "decode_ms_per_step": round(step_s * 1000, 2),
                "decode_tokens_per_s_at_batch_run": round(b / step_s, 1), "steps_timed": 8,
                "steps_config": S, "api": "saint_llm_inference.greedy_decode_cached + KVCacheBundle"}
    full_s = prefill_s + S * step_s
    if b == want_b and full_s <= budget:
        ids = torch.randint(0, cfg.vocab_size, (b, P), device=dev)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            greedy_decode_cached(model, ids, max_new_tokens=S)
            e1.record()
            torch.cuda.synchronize(dev)
        total = e0.elapsed_time(e1) / 1000.0
        dec = max(total - prefill_s, 1e-6)
        return {"metric": "decode tok/s", "value": b * (S - 1) / dec, "unit": "tokens/s",
                "prefill_tokens_per_s": b * P / prefill_s, "n_gpus": 1, "measured": measured,
                "timing": "CUDA events; decode = full call minus the measured prefill"}
    why = (f"prefill at batch {want_b} ran out of memory" if b != want_b else
           f"{S} steps take ~{full_s:.0f} s, over the {budget:.0f} s decode budget")
    return {"unavailable": f"reference decode: {why}; timed at batch {b}, {8} steps", "measured": measured}


def _max_over_ranks(x: float, dev: torch.device, world: int) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _param_count(SaintLLM, cfg) -> int:  # noqa: N803
    with torch.device("meta"):
        return sum(p.numel() for p in SaintLLM(cfg).parameters())


def _run(args) -> dict:
    t_arm = time.perf_counter()
    budget = float(os.environ.get("SV4_REF_BUDGET_S", "600"))
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
    dog = _watchdog(float(os.environ.get("SV4_REF_WATCHDOG_S", "720")), rank) if world > 1 else None
    if world > 1:
        # no NVLink multicast objects: a rank stopped by the driver's time limit must not leave
        # peers' memory bound to one
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)
    try:
        return _run_on_device(args, SaintLLM, ModelConfig, Muon, split_for_muon_adamw, make_loss_fn, rank, world,
                              dev, t_arm, budget)
    finally:
        if dog is not None:
            dog.cancel()
        if world > 1:
            torch.distributed.destroy_process_group()


STAGE = {"name": "start"}


def _stage(name: str) -> None:
    STAGE["name"] = name


def _watchdog(limit_s: float, rank: int) -> threading.Timer:
    """After ``limit_s`` seconds: rank 0 prints the unavailable line with the stage reached,
    then the process exits (every rank runs its own timer from the same start)."""
    def fire() -> None:
        if rank == 0:
            print(json.dumps(_unavailable(f"reference probe did not finish within {limit_s:.0f} s "
                                          f"(stage reached: {STAGE['name']})")), flush=True)
        sys.stdout.flush()
        os._exit(0)

    t = threading.Timer(limit_s, fire)
    t.daemon = True
    t.start()
    return t


def _run_on_device(args, SaintLLM, ModelConfig, Muon, split_for_muon_adamw, make_loss_fn,  # noqa: N803
                   rank, world, dev, t_arm, budget) -> dict:
    cfg = _reference_config(ModelConfig, args)
    full_layers = cfg.n_layers
    have = torch.cuda.get_device_properties(dev).total_memory
    # fp32 weights + grads + Muon momentum per GPU (the AdamW share is small)
    n_params = _param_count(SaintLLM, cfg)
    need = n_params * 12 / world
    fits = need <= 0.9 * have
    cuts = [full_layers]
    if world > 1:
        # FSDP2 shards the fp32 state, but the reference's per-layer working set stays ~135 GB
        # per GPU (measured on one GPU: 167 GB peak at a 4-layer cut holding ~33 GB of state),
        # so the state may take what is left; every rank picks the same cut (no OOM retries:
        # ranks would have to agree on them)
        per_layer = (n_params - _param_count(SaintLLM, _reference_config(ModelConfig, args, 1))) / max(
            full_layers - 1, 1)
        base = n_params - per_layer * full_layers
        budget_params = max(0.0, (have - 150e9)) * world / 12
        run = int(max(1, min(full_layers, (budget_params - base) // per_layer)))
        fits = run == full_layers
        cuts = [run]
    elif not fits:
        # layer cuts whose fp32 state takes at most a third of the memory (the reference's
        # activations and optimizer temporaries take the rest: 133 GB at 2 layers and 2 x 4096
        # tokens); on an out-of-memory error the next smaller cut is tried.  The measured
        # micro-batch time scales linearly to the full depth.
        per_layer = (n_params - _param_count(SaintLLM, _reference_config(ModelConfig, args, 1))) / max(
            full_layers - 1, 1)
        base = n_params - per_layer * full_layers
        top = int(max(1, min(full_layers, (have * world / 36 - base) // per_layer)))
        cuts = sorted({top, max(1, top // 2), max(1, top // 4), 2, 1}, reverse=True)
    last_err = None
    for run_layers in cuts:
        try:
            return _measure(args, SaintLLM, ModelConfig, Muon, split_for_muon_adamw, make_loss_fn, rank, world, dev,
                            t_arm, budget, run_layers, full_layers, fits, n_params, need, have)
        except torch.OutOfMemoryError as e:  # only the one-GPU layer-cut probe retries
            if fits or world > 1:
                raise
            last_err = str(e).splitlines()[0][:120]  # keep no traceback: it would pin the model
        import gc

        gc.collect()
        torch.cuda.empty_cache()
    raise RuntimeError(f"every layer cut ran out of memory ({last_err})")


def _probe_fsdp(args, micro, toks, n_micro, rank, world, dev, t_arm, run_layers, full_layers, n_params, need,
                have) -> dict:
    """N > 1: time one micro-batch under FSDP2 and report it with a lower bound of the step.  The
    optimizer step is not run: the reference's Muon orthogonalises FSDP2 DTensor shards with
    per-operation collectives, and a probe that included one such step did not finish within
    600 s on 2 x B200 (the driver would kill the arm before it printed anything)."""
    _stage("timed micro-batch")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    micro(toks, min(1, n_micro - 1))
    ev[1].record()
    torch.cuda.synchronize()
    mb_ms = _max_over_ranks(ev[0].elapsed_time(ev[1]), dev, world)
    elapsed = _max_over_ranks(time.perf_counter() - t_arm, dev, world)
    scale = full_layers / run_layers
    low_ms = n_micro * mb_ms * scale
    tokens = world * args.seqs_per_gpu * args.seq_len
    measured = {
        "layers_run": run_layers, "layers_config": full_layers, "micro_batch_tokens": args.micro_batch * args.seq_len,
        "micro_batch_ms": round(mb_ms, 1), "micro_batches_per_step": n_micro,
        "step_ms_lower_bound": round(low_ms, 1),
        "tokens_per_s_upper_bound": round(tokens / (low_ms / 1000.0), 1),
        "extrapolation": "micro-batches only (no optimizer step), linear in layers" if scale != 1 else
                         "micro-batches only (no optimizer step)",
        "n_gpus": world, "parallelism": f"fsdp2 dp{world}",
        "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1), "elapsed_s": round(elapsed, 1),
    }
    return _unavailable(
        f"reference under FSDP2 ({need / 1e9:.0f} GB fp32 state per GPU, {run_layers} of {full_layers} layers "
        f"timed): its Muon step over DTensor shards did not finish within the 600 s arm budget on 2 GPUs, so "
        f"only the micro-batch is timed", measured) if rank == 0 else {}


def _measure(args, SaintLLM, ModelConfig, Muon, split_for_muon_adamw, make_loss_fn,  # noqa: N803
             rank, world, dev, t_arm, budget, run_layers, full_layers, fits, n_params, need, have) -> dict:
    cfg = _reference_config(ModelConfig, args, run_layers)
    _stage(f"building the {run_layers}-layer model")
    torch.cuda.reset_peak_memory_stats(dev)
    torch.manual_seed(0)
    with torch.device(dev):
        model = SaintLLM(cfg)
    if world > 1:
        from saint_llm_distributed.fsdp import fsdp2_wrap, init_default_mesh

        # the reference's production setting: a CUDA device mesh over the NCCL group (its
        # default mesh is "cpu", for its gloo tests)
        model = fsdp2_wrap(model, mesh=init_default_mesh(device="cuda"))
    muon_params, adamw_params = split_for_muon_adamw(model)
    muon = Muon(muon_params, lr=2.7e-4)
    adamw = torch.optim.AdamW(adamw_params, lr=2.7e-4, betas=(0.9, 0.95), eps=1e-20, weight_decay=0.1)
    loss_fn = make_loss_fn(cfg.mtp, moe_cfg=cfg.moe)
    n_micro = args.seqs_per_gpu // args.micro_batch
    g = torch.Generator().manual_seed(rank)
    host = torch.randint(0, cfg.vocab_size, (n_micro, args.micro_batch, args.seq_len), generator=g).pin_memory()

    def micro(toks: torch.Tensor, i: int) -> torch.Tensor:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = loss_fn(model, toks[i]).float() / n_micro
        loss.backward()
        return loss.detach()

    def opt_step() -> None:
        muon.step()
        adamw.step()
        muon.zero_grad(set_to_none=True)
        adamw.zero_grad(set_to_none=True)

    def step() -> torch.Tensor:
        total = torch.zeros((), device=dev)
        toks = host.to(dev, non_blocking=True)
        for i in range(n_micro):
            total += micro(toks, i)
        opt_step()
        return total

    # --- probe: one untimed micro-batch, one timed micro-batch, one timed optimizer step
    toks = host.to(dev, non_blocking=True)
    _stage("first (untimed) micro-batch")
    micro(toks, 0)
    torch.cuda.synchronize()
    if world > 1:
        return _probe_fsdp(args, micro, toks, n_micro, rank, world, dev, t_arm, run_layers, full_layers, n_params,
                           need, have)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    micro(toks, min(1, n_micro - 1))
    ev[1].record()
    opt_step()
    ev[2].record()
    torch.cuda.synchronize()
    scale = full_layers / run_layers
    mb_ms = _max_over_ranks(ev[0].elapsed_time(ev[1]), dev, world)
    opt_ms = _max_over_ranks(ev[1].elapsed_time(ev[2]), dev, world)
    est_step_ms = (n_micro * mb_ms + opt_ms) * scale
    elapsed = _max_over_ranks(time.perf_counter() - t_arm, dev, world)
    tokens = world * args.seqs_per_gpu * args.seq_len
    measured = {
        "layers_run": run_layers, "layers_config": full_layers, "micro_batch_tokens": args.micro_batch * args.seq_len,
        "micro_batch_ms": round(mb_ms, 1), "optimizer_step_ms": round(opt_ms, 1),
        "micro_batches_per_step": n_micro, "extrapolated_step_ms": round(est_step_ms, 1),
        "extrapolated_tokens_per_s": round(tokens / (est_step_ms / 1000.0), 1),
        "extrapolation": "linear in layers" if scale != 1 else "micro-batches x measured micro-batch + optimizer",
        "n_gpus": world, "parallelism": f"fsdp2 dp{world}" if world > 1 else "single-gpu",
        "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1), "elapsed_s": round(elapsed, 1),
    }
    if not fits:
        why = (f"reference keeps fp32 weights, grads and Muon momentum: {n_params / 1e9:.1f}B params x 12 B / "
               f"{world} GPU(s) = {need / 1e9:.0f} GB > {have / 1e9:.0f} GB per GPU" if world == 1 else
               f"reference under FSDP2: {need / 1e9:.0f} GB of fp32 state per GPU plus its ~135 GB per-GPU "
               f"working set exceed {have / 1e9:.0f} GB")
        return _unavailable(f"{why}; micro-batches timed on a {run_layers}-layer cut", measured) if rank == 0 else {}
    remaining = (args.warmup + args.steps) * est_step_ms / 1000.0
    if elapsed + remaining > budget:
        return _unavailable(
            f"reference step of {n_micro} x {args.micro_batch * args.seq_len} tokens takes ~{est_step_ms / 1000:.0f} s "
            f"(measured micro-batch + optimizer); {args.warmup}+{args.steps} steps exceed the {budget:.0f} s budget",
            measured) if rank == 0 else {}

    for _ in range(args.warmup):
        step()
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
    ms = _max_over_ranks(start.elapsed_time(end) / args.steps, dev, world)
    final_loss = float(loss.item())
    res = {
        "impl": "reference", "metric": METRIC,
        "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if args.linear_quant == "bf16" else "fp8",
        "data": "synthetic uniform-random tokens; random-init weights N(0,0.02)",
        "config": {"model": "reference SaintLLM, BASELINE config 3 architecture", "n_layers": cfg.n_layers,
                   "global_batch": world * args.seqs_per_gpu, "seq_len": args.seq_len,
                   "parallelism": f"fsdp2 dp{world}" if world > 1 else "single-gpu",
                   "reference_settings": "fp32 params + bf16 autocast, activation checkpointing, "
                                         "per-expert modules",
                   "final_loss": final_loss},
        "measured": measured,
    }
    return res if rank == 0 else {}

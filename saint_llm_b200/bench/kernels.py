"""Microbenchmarks of the native kernels with roofline fractions.

    python -m saint_llm_b200.bench.kernels gemm --m 8192 --n 8192 --k 8192
    python -m saint_llm_b200.bench.kernels attention --t 4096 --heads 16 --mode csa
    python -m saint_llm_b200.bench.kernels moe --tokens 4096 --dim 2048 --inter 1408 --experts 64 --topk 6
    python -m saint_llm_b200.bench.kernels rmsnorm --rows 4096 --dim 2048
    python -m saint_llm_b200.bench.kernels mhc --tokens 4096 --dim 2048 --hc 4
    python -m saint_llm_b200.bench.kernels indexer --t 4096 --index-heads 64 --index-dim 128 --index-m 4
    python -m saint_llm_b200.bench.kernels fp8 --m 16384 --n 2048 --k 2048

Timing: CUDA events on the launching stream around ``--iters`` launches after
``--warmup`` launches, with an L2 flush (a write larger than the 126 MB L2) before every
timed launch, excluded from the timing.  Achieved rates are algorithmic FLOPs or bytes over
the measured time, reported as a fraction of the peaks in ``MEASURED_PEAKS.json`` at the
repository root ("of measured") or of a fixed fallback (6.65 TB/s, 1.59 PFLOP/s) when the
file is absent.  FP8 tensor work is reported against twice the measured bf16 rate (the
dense FP8 rate of the part is twice its bf16 rate).  ``--launches N`` runs N launches and exits (for profiler captures).
"""

from __future__ import annotations

import argparse
import json
import os
from collections.abc import Callable

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks() -> tuple[float, float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "of measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "of fallback"


def timeit(fn: Callable[[], object], *, warmup: int, iters: int) -> float:
    """Median milliseconds per launch, L2 flushed before each timed launch."""
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def report(name: str, ms: float, *, flops: float = 0.0, bytes_: float = 0.0, peak_mult: float = 1.0) -> dict:
    hbm, tf, tag = peaks()
    tf *= peak_mult
    if peak_mult != 1.0:
        tag = f"{tag} x{peak_mult:g}"
    out = {"kernel": name, "ms": round(ms, 4)}
    if flops:
        out["tflops"] = round(flops / ms / 1e9, 1)
        out["tensor_frac"] = f"{flops / ms / 1e9 / tf:.3f} {tag}"
    if bytes_:
        out["gbs"] = round(bytes_ / ms / 1e6, 1)
        out["hbm_frac"] = f"{bytes_ / ms / 1e6 / hbm:.3f} {tag}"
    if flops and bytes_:
        t_roof = max(flops / (tf * 1e9), bytes_ / (hbm * 1e6))
        out["roofline_frac"] = f"{t_roof / ms:.3f} {tag}"
    print(json.dumps(out))
    return out


def _run(args: argparse.Namespace, name: str, fn: Callable[[], object], **cost: float) -> None:
    if args.launches:
        for _ in range(args.launches):
            fn()
        torch.cuda.synchronize()
        return
    report(name, timeit(fn, warmup=args.warmup, iters=args.iters), **cost)


def bench_gemm(args: argparse.Namespace) -> None:
    from saint_llm_b200.ops import gemm

    m, n, k = args.m, args.n, args.k
    if args.wgrad:  # weight-gradient layout: dW (m, n) += dY^T X with the tokens (k) as reduction
        dy = torch.randn(k, m, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(k, n, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(m, n, device="cuda", dtype=torch.float32)
        _run(args, f"gemm_wgrad_acc {m}x{n}x{k}", lambda: gemm.gemm_nt(dy.t(), x.t(), out=acc, accumulate=True),
             flops=2.0 * m * n * k, bytes_=2.0 * (m * k + n * k) + 8.0 * m * n)
        return
    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _run(args, f"gemm_bf16 {m}x{n}x{k}", lambda: gemm.gemm_nt(a, b, out=out),
         flops=2.0 * m * n * k, bytes_=2.0 * (m * k + n * k + m * n))


def bench_fp8(args: argparse.Namespace) -> None:
    """Block-scaled FP8: activation / weight quantisation and the tcgen05 block-scaled GEMM,
    with the bf16 GEMM of the same shape for comparison."""
    from saint_llm_b200.ops import fp8, gemm

    m, n, k = args.m, args.n, args.k
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02
    a, b = fp8.quantize_rows(x), fp8.quantize_blocks(w)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    err = gemm.error_word(torch.device("cuda"))
    ext = __import__("saint_llm_b200.ops.backend", fromlist=["ext"]).ext()
    if args.launches:
        _run(args, "gemm_fp8", lambda: ext.gemm_fp8(a.q, a.sf, b.q, b.sf, out, err))
        return
    _run(args, f"fp8_quant_rows {m}x{k}", lambda: ext.fp8_quant_rows(x, a.q, a.sf, a.scale),
         bytes_=2.0 * m * k + m * k + 4.0 * m * k / 128)
    _run(args, f"fp8_quant_blocks {n}x{k}", lambda: ext.fp8_quant_blocks(w, b.q, b.sf, b.scale),
         bytes_=2.0 * n * k + n * k)
    _run(args, f"gemm_fp8 {m}x{n}x{k}", lambda: ext.gemm_fp8(a.q, a.sf, b.q, b.sf, out, err),
         flops=2.0 * m * n * k, bytes_=1.0 * (m * k + n * k) + 2.0 * m * n, peak_mult=2.0)
    xb = x.clone()
    _run(args, f"gemm_bf16 {m}x{n}x{k}", lambda: gemm.gemm_nt(xb, w, out=out),
         flops=2.0 * m * n * k, bytes_=2.0 * (m * k + n * k + m * n))
    gemm.check_errors(torch.device("cuda"))


def bench_attention(args: argparse.Namespace) -> None:
    from saint_llm_b200.ops import backend, gemm
    from saint_llm_b200.ops.attention import fused_attention

    t, h, d, w = args.t, args.heads, args.head_dim, args.window
    mode = {"swa": 0, "hca": 1, "csa": 2}[args.mode]
    m = {"swa": 1, "hca": 128, "csa": 4}[args.mode]
    n = t // m if mode else 0
    q = torch.randn(1, t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(1, t, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(1, t, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    kv = torch.randn(1, n, d, device="cuda", dtype=torch.bfloat16, requires_grad=True) if mode else None
    sink = torch.zeros(h, device="cuda", requires_grad=True)
    sel = None
    keys_c = 0.0
    if mode == 2:  # indexer picks: half of the causally visible entries
        qpos = torch.arange(t, device="cuda").view(-1, 1)
        causal = (torch.arange(n, device="cuda") * m + m - 1).view(1, -1) < qpos
        pick = causal & (torch.rand(t, n, device="cuda") < 0.5)
        top = torch.where(pick, torch.arange(n, device="cuda").expand(t, n), -1).unsqueeze(0).contiguous()
        sel = torch.empty(1, t, (n + 31) // 32, dtype=torch.int32, device="cuda")
        backend.ext().csa_select_mask(top, n, sel, gemm.error_word(top.device))
        keys_c = float(pick.sum())
    elif mode == 1:  # entry j visible to query i iff j*m + m - 1 < i
        keys_c = float(sum(min(n, i // m) for i in range(t)))
    keys_w = float(sum(min(w, i + 1) for i in range(t)))
    fwd_flops = 4.0 * h * d * (keys_w + keys_c)  # QK^T and PV over visible pairs
    io = 2.0 * (2 * t * h * d + 2 * t * d + n * d)

    def fwd():
        return fused_attention(q, k, v, window=w, sink=sink, softcap=None, kv=kv, mode=mode, m=m, sel=sel)

    if args.backward:
        out = fwd()
        g = torch.randn_like(out)
        _run(args, f"attention_bwd {args.mode} T={t} H={h} d={d}",
             lambda: torch.autograd.grad(out, [q, k, v], g, retain_graph=True),
             flops=2.5 * fwd_flops, bytes_=2 * io)
    else:
        with torch.no_grad():
            _run(args, f"attention_fwd {args.mode} T={t} H={h} d={d}", fwd, flops=fwd_flops, bytes_=io)


def bench_moe(args: argparse.Namespace) -> None:
    from saint_llm_b200.ops.moe import GroupedSwiGLUExperts
    from saint_llm_b200.ops.moe_native import routed_experts

    tok, dim, inter, e, k = args.tokens, args.dim, args.inter, args.experts, args.topk
    experts = GroupedSwiGLUExperts(dim, inter, e, device=torch.device("cuda"), dtype=torch.bfloat16)
    for p in experts.parameters():
        torch.nn.init.normal_(p, std=0.02)
    if args.fp8:  # the training forward on block-scaled FP8 (cached weight copies)
        experts.linear_quant = "fp8"
        experts.fp8_weight_cache = "always"
    x = torch.randn(tok, dim, device="cuda", dtype=torch.bfloat16)
    idx = torch.stack([torch.randperm(e, device="cuda")[:k] for _ in range(tok)])
    w = torch.softmax(torch.randn(tok, k, device="cuda"), -1)
    flops = 2.0 * tok * k * 3 * dim * inter
    with torch.no_grad():
        _run(args, f"moe_routed_fwd{'_fp8' if args.fp8 else ''} T={tok} D={dim} I={inter} E={e} k={k}",
             lambda: routed_experts(x, idx, w, experts), flops=flops, peak_mult=2.0 if args.fp8 else 1.0,
             bytes_=2.0 * (3 * e * dim * inter + 2 * tok * dim))


def bench_rmsnorm(args: argparse.Namespace) -> None:
    from saint_llm_b200.ops.norm import rms_norm

    x = torch.randn(args.rows, args.dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    wt = torch.ones(args.dim, device="cuda", requires_grad=True)
    if args.backward:
        y = rms_norm(x, wt, 1e-6)
        g = torch.randn_like(y)
        _run(args, f"rmsnorm_bwd {args.rows}x{args.dim}",
             lambda: torch.autograd.grad(y, [x, wt], g, retain_graph=True), bytes_=6.0 * args.rows * args.dim)
    else:
        with torch.no_grad():
            _run(args, f"rmsnorm_fwd {args.rows}x{args.dim}", lambda: rms_norm(x, wt, 1e-6),
                 bytes_=4.0 * args.rows * args.dim)


def bench_mhc(args: argparse.Namespace) -> None:
    from saint_llm_b200.config import MHCConfig
    from saint_llm_b200.models.mhc import MHC
    from saint_llm_b200.ops.mhc import mhc_split

    torch.manual_seed(0)
    m = MHC(args.dim, MHCConfig(expansion_factor=args.hc)).cuda()
    x = torch.randn(1, args.tokens, args.hc, args.dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    bytes_ = 2.0 * args.tokens * args.hc * args.dim + 2.0 * args.tokens * args.dim
    if args.backward:
        outs = mhc_split(m, x)
        gs = [torch.randn_like(o) for o in outs]
        _run(args, f"mhc_split_bwd T={args.tokens} n={args.hc} D={args.dim}",
             lambda: torch.autograd.grad(outs, [x], gs, retain_graph=True), bytes_=2 * bytes_)
    else:
        with torch.no_grad():
            _run(args, f"mhc_split_fwd T={args.tokens} n={args.hc} D={args.dim}", lambda: mhc_split(m, x),
                 bytes_=bytes_)


def bench_indexer(args: argparse.Namespace) -> None:
    """Lightning-indexer scores: FLOPs of the visible (block-causal) tiles only."""
    from saint_llm_b200.ops import backend
    from saint_llm_b200.ops.gemm import error_word

    torch.manual_seed(0)
    T, nh, c, m = args.t, args.index_heads, args.index_dim, args.index_m
    nb = T // m
    q = torch.randn(1, T, nh * c, device="cuda", dtype=torch.bfloat16)
    keys = torch.randn(1, nb, c, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(1, T, nh, device="cuda")
    out = torch.empty(1, T, nb, device="cuda")
    err = error_word(torch.device("cuda"))
    vis_tiles = sum(1 for qt in range(0, T, 128) for bt in range(0, nb, 128)
                    if bt * m + m - 1 < min(T, qt + 128) - 1)
    flops = 2.0 * vis_tiles * 128 * 128 * nh * c
    bytes_ = 2.0 * (T * nh * c + nb * c) + 4.0 * (T * nh + T * nb)
    _run(args, f"indexer_scores T={T} heads={nh} c={c} blocks={nb}",
         lambda: backend.ext().indexer_scores(q, keys, w, None, m, 0, out, err), flops=flops, bytes_=bytes_)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("kernel", choices=["gemm", "attention", "moe", "rmsnorm", "mhc", "indexer", "fp8"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--launches", type=int, default=0, help="run N launches and exit (profiler captures)")
    ap.add_argument("--backward", action="store_true")
    ap.add_argument("--fp8", action="store_true", help="moe: block-scaled FP8 forward")
    ap.add_argument("--wgrad", action="store_true", help="gemm: weight-gradient layout with fp32 accumulate")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--t", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--window", type=int, default=128)
    ap.add_argument("--mode", choices=["swa", "hca", "csa"], default="csa")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--dim", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=1408)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=6)
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--hc", type=int, default=4, help="mHC expansion factor")
    ap.add_argument("--index-heads", type=int, default=64)
    ap.add_argument("--index-dim", type=int, default=128)
    ap.add_argument("--index-m", type=int, default=4)
    args = ap.parse_args(argv)
    {"gemm": bench_gemm, "attention": bench_attention, "moe": bench_moe, "rmsnorm": bench_rmsnorm,
     "mhc": bench_mhc, "indexer": bench_indexer, "fp8": bench_fp8}[args.kernel](args)


if __name__ == "__main__":
    main()

"""Prefill and greedy-decode throughput with the heterogeneous KV cache (benchmark
configuration 5 on one GPU: the config-3 architecture, batch 64, 4096-token synthetic
prompts, 512 greedy steps; random-init bf16 weights).

    python -m saint_llm_b200.bench.decode [--batch 64] [--prompt 4096] [--steps 512]

The prompt is prefilled in chunks through the cached forward (every layer's window K/V,
compressed blocks and indexer keys go into the cache).  Decoding (default) imports the
cache into ``infer.static_decode.StaticDecoder`` and replays one CUDA graph per token
(all 28 layers, LM head and argmax, position on the device); ``--engine cached`` feeds
each token through the eager cached forward instead.  Prefill and decode are timed separately with CUDA events after a
synchronize on both sides.  Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=512)
    ap.add_argument("--chunk", type=int, default=256)
    ap.add_argument("--layers", type=int, default=0, help="(development only) override n_layers")
    ap.add_argument("--fp8-experts", action="store_true",
                    help="routed experts on block-scaled FP8 weights (quantised once before the prefill)")
    ap.add_argument("--engine", choices=["graph", "cached"], default="graph",
                    help="graph: static-shape step captured in a CUDA graph; cached: the eager cached path")
    args = ap.parse_args()
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.infer.generate import last_logits
    from saint_llm_b200.infer.kv_cache import KVCacheBundle
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.engine import cast_params

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    upd = {"linear_quant": "bf16"}
    if args.layers:
        upd["n_layers"] = args.layers
    cfg = ModelConfig.bench_16b().model_copy(update=upd)
    torch.manual_seed(0)
    with torch.device(dev):
        model = SaintLLM(cfg)
    cast_params(model, torch.bfloat16)
    model.eval()
    if args.fp8_experts:
        from saint_llm_b200.ops.moe_native import enable_fp8_experts

        enable_fp8_experts(model)
    B, P, S = args.batch, args.prompt, args.steps
    ids = torch.randint(0, cfg.vocab_size, (B, P), device=dev)
    bundle = KVCacheBundle.for_model(model, max_seq_len=P + S, batch_size=B, device=dev)
    out = torch.empty(B, S, dtype=torch.long, device=dev)

    def ev() -> torch.cuda.Event:
        return torch.cuda.Event(enable_timing=True)

    with torch.no_grad():
        torch.cuda.synchronize()
        s0, s1, s2 = ev(), ev(), ev()
        s0.record()
        logits = None
        for c in range(0, P, args.chunk):
            logits = last_logits(model, ids[:, c:c + args.chunk], bundle=bundle)
        s1.record()
        torch.cuda.synchronize()
        prefill_ms = s0.elapsed_time(s1)
        kv_gb = bundle.nbytes() / 1e9
        if args.engine == "cached":
            tok = logits.argmax(-1, keepdim=True)
            for i in range(S):
                out[:, i:i + 1] = tok
                tok = last_logits(model, tok, bundle=bundle).argmax(-1, keepdim=True)
            s2.record()
        else:
            from saint_llm_b200.infer.static_decode import StaticDecoder

            dec = StaticDecoder(model, B, P + S)
            dec.load(bundle, logits)
            del bundle
            dec.capture()  # capture cost is outside the timed decode
            torch.cuda.synchronize()
            s1.record()
            dec.generate(S, out)
            s2.record()
        torch.cuda.synchronize()
    check_errors(dev)
    decode_ms = s1.elapsed_time(s2)
    print(json.dumps({
        "bench": "decode", "metric": "decode tok/s", "value": B * S / (decode_ms / 1000.0), "unit": "tokens/s",
        "prefill_tokens_per_s": B * P / (prefill_ms / 1000.0), "decode_ms_per_step": decode_ms / S,
        "n_gpus": 1, "dtype": "bf16 + fp8 routed experts" if args.fp8_experts else "bf16",
        "data": "synthetic uniform-random prompts; random-init weights",
        "config": {"model": "config-3 architecture (d2048 L%d, 64 routed top-6)" % cfg.n_layers, "batch": B,
                   "prompt": P, "decode_steps": S, "prefill_chunk": args.chunk,
                   "kv_cache_gb": round(kv_gb, 2), "engine": args.engine,
                   "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)},
    }), flush=True)


if __name__ == "__main__":
    main()

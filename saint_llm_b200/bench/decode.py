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


def measure_decode(*, batch: int = 64, prompt: int = 4096, steps: int = 512, chunk: int = 256, layers: int = 0,
                   fp8_experts: bool = False, engine: str = "graph", device: torch.device | None = None,
                   seed: int = 0) -> dict:
    """Prefill + greedy decode throughput of the config-3 architecture on one GPU (random
    init).  Returns tokens/s of both phases and the settings (CUDA-event timed)."""
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.infer.generate import last_logits
    from saint_llm_b200.infer.kv_cache import KVCacheBundle
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.engine import cast_params

    dev = device or torch.device("cuda", torch.cuda.current_device())
    upd = {"linear_quant": "bf16"}
    if layers:
        upd["n_layers"] = layers
    cfg = ModelConfig.bench_16b().model_copy(update=upd)
    torch.manual_seed(seed)
    with torch.device(dev):
        model = SaintLLM(cfg)
    cast_params(model, torch.bfloat16)
    model.eval()
    if fp8_experts:
        from saint_llm_b200.ops.moe_native import enable_fp8_experts

        enable_fp8_experts(model)
    B, P, S = batch, prompt, steps
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g).to(dev)
    bundle = KVCacheBundle.for_model(model, max_seq_len=P + S, batch_size=B, device=dev)
    out = torch.empty(B, S, dtype=torch.long, device=dev)

    def ev() -> torch.cuda.Event:
        return torch.cuda.Event(enable_timing=True)

    with torch.no_grad():
        torch.cuda.synchronize(dev)
        s0, s1, s2 = ev(), ev(), ev()
        s0.record()
        logits = None
        for c in range(0, P, chunk):
            logits = last_logits(model, ids[:, c:c + chunk], bundle=bundle)
        s1.record()
        torch.cuda.synchronize(dev)
        prefill_ms = s0.elapsed_time(s1)
        kv_gb = bundle.nbytes() / 1e9
        if engine == "cached":
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
            torch.cuda.synchronize(dev)
            s1.record()
            dec.generate(S, out)
            s2.record()
        torch.cuda.synchronize(dev)
    check_errors(dev)
    decode_ms = s1.elapsed_time(s2)
    res = {
        "value": B * S / (decode_ms / 1000.0), "unit": "tokens/s",
        "prefill_tokens_per_s": B * P / (prefill_ms / 1000.0), "decode_ms_per_step": decode_ms / S,
        "dtype": "bf16 + fp8 routed experts" if fp8_experts else "bf16",
        "config": {"model": "config-3 architecture (d2048 L%d, 64 routed top-6)" % cfg.n_layers, "batch": B,
                   "prompt": P, "decode_steps": S, "prefill_chunk": chunk, "kv_cache_gb": round(kv_gb, 2),
                   "engine": engine, "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)},
    }
    del model, out
    torch.cuda.empty_cache()
    return res


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
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = measure_decode(batch=args.batch, prompt=args.prompt, steps=args.steps, chunk=args.chunk, layers=args.layers,
                         fp8_experts=args.fp8_experts, engine=args.engine, device=dev)
    print(json.dumps({"bench": "decode", "metric": "decode tok/s", "n_gpus": 1,
                      "data": "synthetic uniform-random prompts; random-init weights", **res}), flush=True)


if __name__ == "__main__":
    main()

"""The CUDA-graph training step (one captured micro-batch replayed per micro-batch)
trains like the eager step (routing pinned): the same losses over three steps; the same
accumulated gradients in the first step (the captured graph against the eager backward on
identical weights) for every parameter, within the spread of two eager runs (some backward
kernels add partial results with atomics) plus bf16 rounding, floored at a small fraction of
the median gradient norm; and in the later steps for all but a handful of parameters (AdamW
turns a near-zero gradient into a sign-sized update, so a few small bias vectors drift apart
after the first update in any two runs)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(dev, graph, data):
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.launch import build_training

    base = ModelConfig.bench_16b()
    # hash routing in both MoE layers and a CSA top-k above the block count (512 > 128 at
    # T = 512): no discrete choice can flip between runs, so later steps stay comparable
    cfg = base.model_copy(update={"n_layers": 2, "moe": base.moe.model_copy(update={"hash_routed_layers": 2})})
    run = RunConfig(grad_accum=2, micro_batch=1, seq_len=512, cuda_graphs=graph, seed=0)
    job = build_training(cfg, run, dev)
    grads: list[dict] = []
    real_step = job.optimizer.step

    def step_and_record(*a, **k):
        grads.append({n: p.main_grad.detach().float().clone() for n, p in job.model.named_parameters()
                      if getattr(p, "main_grad", None) is not None})
        return real_step(*a, **k)

    job.optimizer.step = step_and_record
    losses = [float(job.step.run_device(d).item()) for d in data]
    torch.cuda.synchronize()
    check_errors(dev)
    assert (job.step._graph is not None) == graph, job.step.graph_error
    del job
    torch.cuda.empty_cache()
    return losses, grads


def test_graph_step_matches_eager(cuda):
    torch.manual_seed(5)
    data = [torch.randint(0, 32768, (2, 1, 512), device=cuda) for _ in range(3)]
    l_e1, g_e1 = _run(cuda, False, data)
    l_e2, g_e2 = _run(cuda, False, data)
    l_g, g_g = _run(cuda, True, data)
    for a, b in zip(l_e1, l_g, strict=True):
        assert abs(a - b) <= 2e-3 * abs(a), (l_e1, l_g)
    for step, (e1, e2, gg) in enumerate(zip(g_e1, g_e2, g_g, strict=True)):
        norms = sorted(v.norm().item() for v in e1.values())
        floor = 0.02 * norms[len(norms) // 2]
        bad = []
        for n, ref in e1.items():
            noise = (ref - e2[n]).norm().item()
            diff = (ref - gg[n]).norm().item()
            if diff > 2 * noise + 0.02 * ref.norm().item() + floor:
                bad.append((n, diff, noise, ref.norm().item()))
        allowed = 0 if step == 0 else max(2, len(e1) // 100)
        assert len(bad) <= allowed, (step, bad[:8])

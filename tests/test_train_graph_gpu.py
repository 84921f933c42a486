"""The CUDA-graph training step (one captured micro-batch replayed per micro-batch)
trains like the eager step: the same losses, and weight updates that differ from the
eager ones no more than two eager runs differ from each other (some backward kernels add
partial results with atomics, so two eager runs are not bit-identical either)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(dev, graph, data):
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.ops.gemm import check_errors
    from saint_llm_b200.train.launch import build_training

    cfg = ModelConfig.bench_16b().model_copy(update={"n_layers": 2})
    run = RunConfig(grad_accum=2, micro_batch=1, seq_len=512, cuda_graphs=graph, seed=0)
    job = build_training(cfg, run, dev)
    w0 = {n: p.detach().float().clone() for n, p in job.model.named_parameters()}
    losses = [float(job.step.run_device(d).item()) for d in data]
    torch.cuda.synchronize()
    check_errors(dev)
    assert (job.step._graph is not None) == graph, job.step.graph_error
    upd = {n: p.detach().float() - w0[n] for n, p in job.model.named_parameters()}
    del job
    torch.cuda.empty_cache()
    return losses, upd


def test_graph_step_matches_eager(cuda):
    torch.manual_seed(5)
    data = [torch.randint(0, 32768, (2, 1, 512), device=cuda) for _ in range(3)]
    l_e1, u_e1 = _run(cuda, False, data)
    l_e2, u_e2 = _run(cuda, False, data)
    l_g, u_g = _run(cuda, True, data)
    for a, b in zip(l_e1, l_g, strict=True):
        assert abs(a - b) <= 2e-3 * abs(a), (l_e1, l_g)
    bad = []
    for n, ue in u_e1.items():
        scale = ue.norm().item() + 1e-12
        noise = (ue - u_e2[n]).norm().item() / scale
        diff = (ue - u_g[n]).norm().item() / scale
        if diff > 2 * noise + 0.05:
            bad.append((n, round(diff, 4), round(noise, 4)))
    assert not bad, bad[:8]

"""The CUDA-graph training step (one captured micro-batch replayed per micro-batch)
trains exactly like the eager step: same losses and the same weights after three steps."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _job(dev, graph):
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.train.launch import build_training

    cfg = ModelConfig.bench_16b().model_copy(update={"n_layers": 2})
    run = RunConfig(grad_accum=2, micro_batch=1, seq_len=512, cuda_graphs=graph, seed=0)
    return build_training(cfg, run, dev)


def test_graph_step_matches_eager(cuda):
    from saint_llm_b200.ops.gemm import check_errors

    torch.manual_seed(5)
    data = [torch.randint(0, 32768, (2, 1, 512), device=cuda) for _ in range(3)]
    losses, weights = {}, {}
    for graph in (False, True):
        job = _job(cuda, graph)
        losses[graph] = [float(job.step.run_device(d).item()) for d in data]
        torch.cuda.synchronize()
        check_errors(cuda)
        assert (job.step._graph is not None) == graph, job.step.graph_error
        weights[graph] = {n: p.detach().float().clone() for n, p in job.model.named_parameters()}
        del job
        torch.cuda.empty_cache()
    for a, b in zip(losses[False], losses[True], strict=True):
        assert abs(a - b) <= 2e-3 * abs(a), (losses[False], losses[True])
    worst = 0.0
    for n, w in weights[False].items():
        d = (w - weights[True][n]).abs().max().item() / (w.abs().max().item() + 1e-6)
        worst = max(worst, d)
    assert worst < 2e-2, worst

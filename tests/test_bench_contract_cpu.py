"""The bench's run layout arithmetic on CPU: the RunConfig it hands ``build_training`` for
each parallel layout, and the uniform-prediction loss it reports next to the measured one."""

import argparse
import importlib.util
import math
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _args(**kw):
    base = dict(micro_batch=4, seqs_per_gpu=32, seq_len=4096, no_zero=False, ep_transport="p2p",
                no_overlap_reduce=False, zero_transport="p2p", no_cuda_graph=False, fp8_expert_cache="auto",
                tp=1, tp_transport="nccl")
    base.update(kw)
    return argparse.Namespace(**base)


def test_run_config_without_tp(bench):
    run = bench.run_config(_args(), 8)
    assert (run.ep, run.tp, run.zero, run.micro_batch, run.grad_accum) == (8, 1, "hybrid_zero", 4, 8)
    assert run.fused_ep and run.fused_zero and run.zero_transport == "p2p" and not run.fused_tp
    plain = bench.run_config(_args(no_zero=True, ep_transport="nccl", no_overlap_reduce=True), 2)
    assert plain.zero == "dp" and not plain.fused_ep and not plain.fused_zero


def test_run_config_with_tp_keeps_the_tokens_per_gpu(bench):
    args = _args(tp=2, tp_transport="p2p")
    run = bench.run_config(args, 8)
    # a TP pair shares batches of 2 x 4 sequences and takes the same 8 micro-batches per step:
    # 64 sequences per pair = 32 per GPU, as without TP
    assert (run.ep, run.tp, run.micro_batch, run.grad_accum) == (8, 2, 8, 8) and run.fused_tp
    assert run.micro_batch * run.grad_accum == args.tp * args.seqs_per_gpu


def test_uniform_loss_counts_the_mtp_heads(bench):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.train.losses import mtp_weight

    cfg = ModelConfig.bench_16b()
    w = 1.0 + sum(mtp_weight(cfg.mtp, k) for k in range(cfg.mtp.depth))
    assert bench._uniform_loss(cfg) == pytest.approx(w * math.log(cfg.vocab_size))
    assert bench._uniform_loss(cfg) > math.log(cfg.vocab_size)

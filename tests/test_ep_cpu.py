"""Expert parallelism on 2 gloo CPU ranks: dispatch/combine round trip and the EP MoE
layer against the same layer with all experts local."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.distributed


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, ws: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.config import MoEConfig
        from saint_llm_b200.models.moe import DeepSeekMoE
        from saint_llm_b200.parallel import ep

        torch.manual_seed(rank)
        tok = torch.randn(10, 4)
        eid = torch.randint(0, 4, (10,))
        plan = ep.dispatch_tokens_by_expert(tok, eid, n_experts=4)
        back = ep.combine_outputs_by_expert(plan.permuted_tokens * 1.0, plan)
        ok_roundtrip = torch.equal(back, tok)

        torch.manual_seed(0)
        cfg = MoEConfig(hash_routed_layers=0, shared_experts=1, routed_experts=4, experts_per_token=2,
                        expert_intermediate_dim=16)
        full = DeepSeekMoE(8, cfg, layer_idx=0, use_grouped_gemm=True)
        local = DeepSeekMoE(8, cfg, layer_idx=0, use_grouped_gemm=True)
        local.load_state_dict(full.state_dict())
        experts = ep.shard_grouped_experts(local, rank, ws, None)
        torch.manual_seed(100 + rank)
        x = torch.randn(1, 6, 8, requires_grad=True)
        y_full = full(x)
        y_ep = local(x)
        ok_fwd = torch.allclose(y_full, y_ep, atol=1e-5)
        y_ep.sum().backward()
        y_full.sum().backward()
        per = 2
        # each rank's local expert grads cover the tokens of every rank: compare to the sum over ranks
        g_sum = full.grouped_experts.down_weight.grad.clone()
        dist.all_reduce(g_sum)
        g_sum = g_sum[rank * per:(rank + 1) * per]
        ok_bwd = torch.allclose(local.grouped_experts.down_weight.grad, g_sum, atol=1e-5)
        q.put((rank, ok_roundtrip, ok_fwd, ok_bwd, len(experts)))
    finally:
        dist.destroy_process_group()


def test_ep_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, rt, fwd, bwd, n in res:
        assert rt and fwd and bwd, (rank, rt, fwd, bwd)
        assert n == 3


def test_dispatch_simulation_mode():
    from saint_llm_b200.parallel import ep

    tok = torch.arange(24.0).view(6, 4)
    eid = torch.tensor([3, 0, 2, 1, 0, 3])
    plan = ep.dispatch_tokens_by_expert(tok, eid, n_experts=4, world_size=2)
    assert plan.simulated and plan.send_counts.tolist() == [3, 3]
    assert torch.equal(ep.combine_outputs_by_expert(plan.permuted_tokens, plan), tok)


def _step_worker(rank: int, ws: int, port: int, zero: bool, q, overlap: bool = False, micro: int = 1) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // ws))  # the ranks share the host's cores
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        import copy

        from saint_llm_b200.config import ModelConfig
        from saint_llm_b200.models import SaintLLM
        from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
        from saint_llm_b200.parallel import ep
        from saint_llm_b200.train.engine import attach_main_grads
        from saint_llm_b200.train.step import TrainStep

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        torch.manual_seed(0)
        ref = SaintLLM(cfg)
        model = copy.deepcopy(ref)
        torch.manual_seed(11)
        data = [torch.randint(0, cfg.vocab_size, (micro, 1, 16)) for _ in range(ws)]
        init = {n: p.detach().clone() for n, p in ref.named_parameters()}
        # reference: one process, the mean of every rank's loss, one optimizer step
        rp = attach_main_grads(ref)
        ropt = MuonAdamW(*split_for_muon_adamw(ref), lr=0.02, qk_clip_enabled=False)
        rstep = TrainStep(ref, ropt, micro_batches=1, params=rp)
        for d in data:
            for i in range(micro):
                (rstep.loss_fn(ref, d[i]) / (ws * micro)).backward()
        ref_grads = {n: p.main_grad.clone() for n, p in ref.named_parameters() if hasattr(p, "main_grad")}
        ropt.step()
        # expert + data parallel with (or without) hybrid ZeRO
        sync = ep.setup_expert_parallel(model, transport="nccl", zero=zero, overlap_reduce=overlap)
        params = attach_main_grads(model)
        opt = MuonAdamW(*split_for_muon_adamw(model), lr=0.02, qk_clip_enabled=False)
        sync.configure_optimizer(opt)
        step = TrainStep(model, opt, micro_batches=micro, params=params, grad_sync=sync)
        grads: dict[str, torch.Tensor] = {}
        real_step = opt.step

        def step_and_record(*a, **k):  # the synchronised gradients the optimizer steps with
            for n, p in model.named_parameters():
                if sync.is_updated_here(p) and hasattr(p, "main_grad"):
                    grads[n] = p.main_grad.clone()
            return real_step(*a, **k)

        opt.step = step_and_record
        step.run_device(data[rank])
        per = cfg.moe.routed_experts // ws
        refp = dict(ref.named_parameters())
        worst, moved = 0.0, 0.0
        g_worst = 0.0
        for n, p in model.named_parameters():
            r, rg = refp[n], ref_grads.get(n)
            if ".grouped_experts." in n:
                r = r[rank * per:(rank + 1) * per]
                rg = rg[rank * per:(rank + 1) * per] if rg is not None else None
            worst = max(worst, float((p.detach() - r.detach()).abs().max()))
            if n in grads and rg is not None:
                # floor: the mHC static biases' gradients are ~1e-7 cancelling sums
                g_worst = max(g_worst, float((grads[n] - rg).abs().max() / rg.abs().max().clamp(min=1e-5)))
        for n, p1 in ref.named_parameters():
            moved = max(moved, float((p1.detach() - init[n]).abs().max()))
        q.put((rank, worst, moved, g_worst, len(grads)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("zero,overlap,micro", [(False, False, 1), (True, False, 1), (True, True, 2)])
def test_ep_dp_step_matches_single_process(zero, overlap, micro):
    """One step of expert + data parallel training (plain, hybrid ZeRO, and hybrid ZeRO
    with the per-block reductions overlapped with the last micro-batch's backward)
    equals one process stepping on the mean of every rank's loss."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_step_worker, args=(r, 2, port, zero, q, overlap, micro)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, worst, moved, g_worst, n_grads in res:
        # the gradients each rank steps with equal the single process's (a wrong averaging
        # factor hides in the weights: Muon and AdamW updates barely depend on the scale)
        assert n_grads > 20 and g_worst < 1e-3, (zero, rank, g_worst, n_grads)
        # the step moved weights by ~`moved`; the parallel step must agree to fp32 noise.
        # Gradient sums run in a different order; parameters whose gradient is a heavily
        # cancelling sum (mHC gate biases) differ by ~0.5 % of their own size, and
        # Newton-Schulz carries that into the update.  A missing reduction, owner or
        # broadcast would differ by ~`moved`.
        assert worst < 1e-2 * max(moved, 1e-3) + 2e-5, (zero, rank, worst, moved)

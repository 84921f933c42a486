"""Tensor parallelism on attention composed with expert parallelism and (hybrid ZeRO) data
parallelism, on 4 gloo CPU ranks (TP=2 x 2 replicas, EP=4): one training step equals one
process stepping on the mean of the replicas' losses."""

import copy
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


def _global_name(n: str, rank: int, per: int) -> str:
    """Local output group i of TP rank r is the full model's group r * per + i."""
    if ".group_projs." not in n:
        return n
    head, tail = n.split(".group_projs.")
    i, rest = tail.split(".", 1)
    return f"{head}.group_projs.{rank * per + int(i)}.{rest}"


def _slice_like(ref: torch.Tensor, p: torch.Tensor, n: str, tp_rank: int, ep_rank: int, e_per: int) -> torch.Tensor:
    if ".grouped_experts." in n:
        return ref[ep_rank * e_per:(ep_rank + 1) * e_per]
    if p.shape == ref.shape:
        return ref
    if n.endswith("q_up.weight") or n.endswith("sink_logit"):
        r = p.shape[0]
        return ref[tp_rank * r:(tp_rank + 1) * r]
    if n.endswith("final_proj.weight"):
        c = p.shape[1]
        return ref[:, tp_rank * c:(tp_rank + 1) * c]
    raise AssertionError(f"unexpected shape for {n}: {tuple(p.shape)} vs {tuple(ref.shape)}")


def _worker(rank: int, ws: int, tp: int, port: int, zero: bool, overlap: bool, micro: int, q,
            nccl: bool = False) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)  # four ranks share the host's cores
    if nccl:  # one GPU per rank, NCCL collectives, the model's math on the eager fp32 path
        import datetime

        from saint_llm_b200.ops import backend

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        ctx = backend.eager_mode(True)
    else:
        import contextlib

        dev = torch.device("cpu")
        dist.init_process_group("gloo", rank=rank, world_size=ws)
        ctx = contextlib.nullcontext()
    ctx.__enter__()
    try:
        from saint_llm_b200.config import ModelConfig
        from saint_llm_b200.models import SaintLLM
        from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
        from saint_llm_b200.parallel.tp_ep import setup_tp_ep
        from saint_llm_b200.train.engine import attach_main_grads
        from saint_llm_b200.train.step import TrainStep

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        torch.manual_seed(0)
        ref = SaintLLM(cfg).to(dev)
        model = copy.deepcopy(ref)
        replicas = ws // tp
        torch.manual_seed(11)
        data = [torch.randint(0, cfg.vocab_size, (micro, 2, 16)).to(dev) for _ in range(replicas)]
        init = {n: p.detach().clone() for n, p in ref.named_parameters()}
        rp = attach_main_grads(ref)
        ropt = MuonAdamW(*split_for_muon_adamw(ref), lr=0.02, qk_clip_enabled=False, ns_impl="reference")
        rstep = TrainStep(ref, ropt, micro_batches=1, params=rp)
        for d in data:
            for i in range(micro):
                (rstep.loss_fn(ref, d[i]) / (replicas * micro)).backward()
        ref_grads = {n: p.main_grad.clone() for n, p in ref.named_parameters() if hasattr(p, "main_grad")}
        ropt.step()

        sync, lay = setup_tp_ep(model, tp, transport="nccl", zero=zero, overlap_reduce=overlap)
        params = attach_main_grads(model)
        opt = MuonAdamW(*split_for_muon_adamw(model), lr=0.02, qk_clip_enabled=False, ns_impl="reference")
        sync.configure_optimizer(opt)
        step = TrainStep(model, opt, micro_batches=micro, params=params, grad_sync=sync)
        # the synchronised gradients, as the optimizer sees them (Muon and AdamW updates are
        # nearly invariant to a gradient's scale, so the weights alone would hide a wrong factor)
        grads: dict[str, torch.Tensor] = {}
        real_step = opt.step

        def step_and_record(*a, **k):
            for n, p in model.named_parameters():
                if sync.is_updated_here(p) and hasattr(p, "main_grad"):
                    grads[n] = p.main_grad.clone()
            return real_step(*a, **k)

        opt.step = step_and_record
        loss = float(step.run_device(data[lay.replica]))
        e_per = cfg.moe.routed_experts // ws
        g_per = cfg.attention.output_proj_groups // tp
        refp = dict(ref.named_parameters())
        worst, moved, n_cmp = 0.0, 0.0, 0
        g_worst = 0.0
        for n, p in model.named_parameters():
            gn = _global_name(n, lay.tp_rank, g_per)
            r = _slice_like(refp[gn], p, n, lay.tp_rank, rank, e_per)
            worst = max(worst, float((p.detach() - r.detach()).abs().max()))
            n_cmp += 1
            if n in grads:
                rg = _slice_like(ref_grads[gn], p, n, lay.tp_rank, rank, e_per)
                # the floor covers gradients that are heavily cancelling sums (the mHC static
                # biases' are ~1e-7): their summation-order noise is ~1e-9 in absolute terms
                g_worst = max(g_worst, float((grads[n] - rg).abs().max() / rg.abs().max().clamp(min=1e-5)))
        for n, p1 in ref.named_parameters():
            moved = max(moved, float((p1.detach() - init[n]).abs().max()))
        heads = model.blocks[0].attention.attn_cfg.query_heads
        q.put((rank, worst, moved, n_cmp, heads, loss, g_worst, len(grads)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        ctx.__exit__(None, None, None)
        dist.destroy_process_group()


@pytest.mark.parametrize("zero,overlap,micro", [(False, False, 1), (True, False, 1), (True, True, 2)])
def test_tp_ep_step_matches_single_process(zero, overlap, micro):
    _check_tp_ep_step(zero, overlap, micro, nccl=False)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_tp_ep_step_over_nccl_on_four_gpus():
    """The same layout with NCCL collectives on four GPUs (TP and EP over NCCL, ZeRO with the
    NCCL transport; NVLS off, as for every multi-GPU test)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    _check_tp_ep_step(True, True, 2, nccl=True)


def _check_tp_ep_step(zero, overlap, micro, *, nccl):
    ws, tp = 4, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, tp, port, zero, overlap, micro, q, nccl)) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 8, r
        rank, worst, moved, n_cmp, heads, loss, g_worst, n_grads = r
        assert heads == 2 and n_cmp > 50 and n_grads > 20
        # every gradient this rank steps with equals the single process's (its slice of it)
        assert g_worst < 1e-3, (zero, overlap, rank, g_worst)
        # as in the EP-only equivalence test: a wrong reduction, scale or slice would differ
        # by about `moved`; different summation orders stay at fp32 noise
        assert worst < 1e-2 * max(moved, 1e-3) + 2e-5, (zero, overlap, rank, worst, moved)
    # the TP ranks of one replica report the same loss
    losses = {r[0]: r[5] for r in res}
    assert abs(losses[0] - losses[1]) < 1e-5 and abs(losses[2] - losses[3]) < 1e-5


def _job_worker(rank: int, ws: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.config import ModelConfig, RunConfig
        from saint_llm_b200.train.launch import build_training

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        run = RunConfig(ep=ws, tp=2, zero="hybrid_zero", fused_ep=False, zero_transport="nccl", grad_accum=1,
                        micro_batch=2, seq_len=16, lr=0.02, adamw_lr=3e-3, param_dtype="float32",
                        compute_dtype="float32")
        job = build_training(cfg, run, torch.device("cpu"))
        torch.manual_seed(100 + job.replica)
        batch = torch.randint(0, cfg.vocab_size, (1, 2, 16))
        losses = [job.step(batch) for _ in range(4)]
        q.put((rank, job.replica, job.replicas, losses))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_build_training_with_tensor_parallelism():
    """``RunConfig(tp=2, ep=4)`` through the public builder: ranks 0-1 and 2-3 form the two
    replicas, each TP pair reports the same losses, and training makes progress."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_job_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(4)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    assert all(len(r) == 4 for r in res), res
    assert [(r[1], r[2]) for r in res] == [(0, 2), (0, 2), (1, 2), (1, 2)]
    for a, b in ((0, 1), (2, 3)):
        assert all(abs(x - y) < 1e-4 for x, y in zip(res[a][3], res[b][3], strict=True))
    for r in res:
        assert r[3][-1] < r[3][0]


def _decode_worker(rank: int, ws: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.config import ModelConfig
        from saint_llm_b200.infer.generate import decode, last_logits
        from saint_llm_b200.infer.sampling import SamplingParams
        from saint_llm_b200.models import SaintLLM
        from saint_llm_b200.parallel.tp_ep import parallel_decode, shard_for_inference

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        torch.manual_seed(0)
        full = SaintLLM(cfg).eval()
        model = copy.deepcopy(full)
        torch.manual_seed(21)
        prompts = torch.randint(0, cfg.vocab_size, (4, 12))
        with torch.no_grad():
            want = decode(full, prompts, max_new_tokens=6, params=SamplingParams(), use_cache=True)
            want_logits = last_logits(full, prompts)
        lay = shard_for_inference(model, 2)
        rows = slice(2 * lay.replica, 2 * lay.replica + 2)
        with torch.no_grad():
            got_logits = last_logits(model, prompts[rows])
            got = parallel_decode(model, prompts[rows], max_new_tokens=6)
            eos = int(got[0, 14])  # a token the first row produces: rows are cut after it
            cut = parallel_decode(model, prompts[rows], max_new_tokens=6, eos_token=eos)
        err = float((got_logits - want_logits[rows]).abs().max() / want_logits.abs().max())
        first = int((cut[0, 12:] == eos).nonzero()[0])
        ok_cut = bool((cut[0, 12 + first:] == eos).all()) and torch.equal(cut[0, :12 + first], got[0, :12 + first])
        q.put((rank, err, torch.equal(got, want[rows]), ok_cut, model.blocks[0].attention.attn_cfg.query_heads))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_tp_ep_decode_matches_single_process():
    """Config 5's layout on 4 gloo ranks (TP=2 x EP=4, 2 replicas): each replica decodes its
    two prompts through the KV cache with head-sharded attention and experts over all ranks;
    prefill logits and greedy tokens equal one process decoding all four prompts."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decode_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 5, r
        rank, err, same_tokens, ok_cut, heads = r
        assert heads == 2 and err < 1e-4 and same_tokens and ok_cut, r


def _state_worker(rank: int, ws: int, port: int, tp: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.config import ModelConfig
        from saint_llm_b200.models import SaintLLM
        from saint_llm_b200.parallel.ep import setup_expert_parallel
        from saint_llm_b200.parallel.state import gather_full_state_dict, load_full_state_dict
        from saint_llm_b200.parallel.tp_ep import setup_tp_ep

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        torch.manual_seed(0)
        model = SaintLLM(cfg)
        want = {k: v.clone() for k, v in model.state_dict().items()}
        if tp > 1:
            setup_tp_ep(model, tp, transport="nccl")
        else:
            setup_expert_parallel(model, transport="nccl")
        sharded_keys = sum(1 for k, v in model.state_dict().items() if v.shape != want.get(k, v).shape)
        got = gather_full_state_dict(model)
        same = set(got) == set(want) and all(torch.equal(got[k], want[k]) for k in want)
        # a different full state loads into the shards and gathers back unchanged
        other = {k: (v + 1 if v.is_floating_point() else v) for k, v in want.items()}
        load_full_state_dict(model, other)
        back = gather_full_state_dict(model)
        same_back = all(torch.equal(back[k], other[k]) for k in other)
        q.put((rank, same, same_back, sharded_keys))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tp", [1, 2])
def test_full_state_dict_round_trip(tp):
    """The unsharded state dict of an EP (tp=1) or TP x EP (tp=2) model on 4 gloo ranks equals
    the model's before sharding, and a full state dict loads back into the shards."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_state_worker, args=(r, 4, port, tp, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 4 and r[1] and r[2], r
        assert r[3] > 0  # something was really sharded


def _ckpt_worker(rank: int, ws: int, port: int, path: str, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.config import ModelConfig, RunConfig
        from saint_llm_b200.parallel.state import gather_full_state_dict
        from saint_llm_b200.train.launch import build_training

        cfg = ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True})
        run = RunConfig(ep=ws, tp=2, zero="hybrid_zero", fused_ep=False, zero_transport="nccl", micro_batch=2,
                        seq_len=16, lr=0.02, adamw_lr=3e-3, param_dtype="float32", compute_dtype="float32")
        torch.manual_seed(100)
        batches = [torch.randint(0, cfg.vocab_size, (1, 2, 16)) for _ in range(2 * (ws // 2))]
        job = build_training(cfg, run, torch.device("cpu"))
        mine = batches[2 * job.replica:2 * job.replica + 2]
        job.step(mine[0])
        job.save(path, step=1)
        after_save = job.step(mine[1])  # the step a resumed run must reproduce
        fresh = build_training(cfg, run.model_copy(update={"seed": 7}), torch.device("cpu"))  # other weights
        step = fresh.load(path)
        resumed = fresh.step(mine[1])
        a, b = gather_full_state_dict(job.model), gather_full_state_dict(fresh.model)
        same = all(torch.allclose(a[k], b[k], atol=1e-6) for k in a)
        q.put((rank, step, abs(after_save - resumed), same))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_training_job_checkpoint_resume(tmp_path):
    """A TP x EP x ZeRO job (4 gloo ranks) saves a sharded checkpoint; a job built with other
    weights loads it and takes the same next step (loss and every weight); the checkpoint's
    model file is the plain single-process state dict."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    path = str(tmp_path / "ckpt")
    procs = [ctx.Process(target=_ckpt_worker, args=(r, 4, port, path, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 4 and r[1] == 1 and r[2] < 1e-5 and r[3], r
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.train.checkpoint import load_checkpoint, sharded_to_v1

    m = SaintLLM(ModelConfig.tiny().model_copy(update={"moe_use_grouped_gemm": True}))
    info = load_checkpoint(sharded_to_v1(path, tmp_path / "v1.pt"), m)
    assert info["step"] == 1

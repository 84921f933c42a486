"""Tensor, context and pipeline parallelism on 2 gloo CPU ranks against the same model
run in one process (fp32)."""

import copy
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.distributed


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, ws=2, nccl=False):
    """Run ``fn(rank, ws)`` on ``ws`` spawned ranks: gloo on CPU, or (``nccl``) one GPU per
    rank over NCCL with the model's math on the eager fp32 path (the comparison against one
    process stays exact; the collectives and p2p exchanges are the real NCCL ones)."""
    ctx = mp.get_context("spawn")
    q, port = ctx.Queue(), _port()
    ps = [ctx.Process(target=_entry, args=(fn, r, ws, port, q, nccl)) for r in range(ws)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(ws)]
    for p in ps:
        p.join(timeout=60)
    return res


DEV = torch.device("cpu")


def _entry(fn, rank, ws, port, q, nccl=False):
    import datetime

    global DEV
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // ws))  # the ranks share the host's cores
    if nccl:
        DEV = torch.device("cuda", rank)
        torch.cuda.set_device(DEV)
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=120),
                                device_id=DEV)
    else:
        dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from saint_llm_b200.ops import backend

        with backend.eager_mode(nccl):
            q.put(fn(rank, ws))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _ids(*shape, vocab):
    return torch.randint(0, vocab, shape).to(DEV)


def _model(**upd):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM

    cfg = ModelConfig.tiny().model_copy(update=upd)
    torch.manual_seed(0)
    return SaintLLM(cfg).to(DEV)


def _close(a, b, tol=2e-4):
    return bool(torch.allclose(a, b, atol=tol, rtol=1e-3))


# ------------------------------------------------------------------ TP
def _tp(rank, ws):
    from saint_llm_b200.parallel.tp import apply_tensor_parallel

    full = _model()
    tp = copy.deepcopy(full)
    sync = apply_tensor_parallel(tp)
    torch.manual_seed(5)
    ids = _ids(2, 24, vocab=full.cfg.vocab_size)
    lf = full(ids)["logits"]
    lf.square().mean().backward()
    lt = tp(ids)["logits"]
    lt.square().mean().backward()
    sync()
    ok = [_close(lt, lf)]
    fp = dict(full.named_parameters())
    per = full.cfg.attention.output_proj_groups // ws
    for n, p in tp.named_parameters():
        if ".group_projs." in n:  # local group i is global group rank * per + i
            head, tail = n.split(".group_projs.")
            i, rest = tail.split(".", 1)
            n = f"{head}.group_projs.{rank * per + int(i)}.{rest}"
        g_full = fp[n].grad
        if p.grad is None or g_full is None:
            continue
        if p.shape == g_full.shape:
            ok.append(_close(p.grad, g_full))
        elif n.endswith("q_up.weight"):
            r = p.shape[0]
            ok.append(_close(p.grad, g_full[rank * r:(rank + 1) * r]))
    return rank, all(ok), len(ok)


def test_tensor_parallel_attention_two_ranks():
    res = _run(_tp)
    for r in res:
        assert r[1] is True and r[2] > 20, r


# ------------------------------------------------------------------ CP
def _cp(rank, ws):
    from saint_llm_b200.parallel.cp import cp_lm_loss

    for pattern in ("csa_hca_interleaved", "nsa", "visual"):
        upd = {"attention_pattern": "csa_hca_interleaved" if pattern == "visual" else pattern}
        if pattern == "nsa":
            from saint_llm_b200.config import NSAConfig

            upd["nsa"] = NSAConfig(compression_rate=8, selection_k=2)
        full = _model(**upd)
        cp = copy.deepcopy(full)
        torch.manual_seed(7)
        ids = _ids(2, 64, vocab=full.cfg.vocab_size)
        if pattern == "visual":  # image tokens on both shards: the indexer's cohesion bias must cross them
            ids[:, 3:9] = full.cfg.tokenizer_slots.image_pad
            ids[:, 40:41] = full.cfg.tokenizer_slots.image_pad
        h, _ = full.backbone(ids)
        logits = full.logits(h).float()
        ref = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
        ref.backward()
        loss = cp_lm_loss(cp, ids)
        loss.backward()
        tot = loss.detach().clone()
        dist.all_reduce(tot)
        if not _close(tot, ref.detach(), 1e-5):
            return rank, f"{pattern}: loss {tot.item()} vs {ref.item()}"
        fp = dict(full.named_parameters())
        for n, p in cp.named_parameters():
            g = p.grad if p.grad is not None else torch.zeros_like(p)
            dist.all_reduce(g)
            ref_g = fp[n].grad if fp[n].grad is not None else torch.zeros_like(p)
            if not _close(g, ref_g):
                return rank, f"{pattern}: grad {n} max err {(g - ref_g).abs().max().item()}"
    return rank, True


def _cp_mtp(rank, ws):
    """The CP training loss with the MTP heads equals the single-process main + MTP loss."""
    from saint_llm_b200.parallel.cp import cp_lm_loss
    from saint_llm_b200.train.losses import cross_entropy_with_mtp

    from saint_llm_b200.config import ModelConfig

    # a large balance weight, so a balance term computed per shard would show in the gradients
    full = _model(moe=ModelConfig.tiny().moe.model_copy(update={"sequence_balance_weight": 0.5}))
    cp = copy.deepcopy(full)
    torch.manual_seed(8)
    ids = _ids(2, 64, vocab=full.cfg.vocab_size)
    ref = cross_entropy_with_mtp(full(ids), ids, cfg=full.cfg.mtp, moe_cfg=full.cfg.moe)
    ref.backward()
    loss = cp_lm_loss(cp, ids, mtp=True, balance=True)
    loss.backward()
    tot = loss.detach().clone()
    dist.all_reduce(tot)
    if not _close(tot, ref.detach(), 1e-5):
        return rank, f"loss {tot.item()} vs {ref.item()}"
    fp = dict(full.named_parameters())
    n = 0
    for name, p in cp.named_parameters():
        g = p.grad if p.grad is not None else torch.zeros_like(p)
        dist.all_reduce(g)
        ref_g = fp[name].grad if fp[name].grad is not None else torch.zeros_like(p)
        if not _close(g, ref_g):
            return rank, f"grad {name} max err {(g - ref_g).abs().max().item()}"
        n += name.startswith("mtp.")
    return rank, n > 0


def test_context_parallel_loss_with_mtp_heads():
    res = _run(_cp_mtp)
    for r in res:
        assert r[1] is True, r


def test_context_parallel_two_ranks():
    res = _run(_cp)
    for r in res:
        assert r[1] is True, r


def _cp_compact(rank, ws):
    """A CP view hands a window layer only the halo plus the local rows, with the halo's global
    start as key_offset; the full-length form (NSA) pads with zeros before the halo."""
    from saint_llm_b200.parallel.cp import CPLayerView

    tl, w, d = 16, 4, 8
    k = torch.full((1, tl, d), float(rank + 1))
    v = -k
    compact = CPLayerView(None, tl, w)
    kc, vc = compact.append(k, v)
    full = CPLayerView(None, tl, w, compact=False)
    kf, _ = full.append(k, v)
    if rank == 0:
        ok = kc.shape[1] == tl and compact.key_offset == 0 and kf.shape[1] == tl
    else:
        ok = (kc.shape[1] == w + tl and compact.key_offset == rank * tl - w and bool((kc[:, :w] == rank).all())
              and bool((vc[:, :w] == -rank).all()) and kf.shape[1] == rank * tl + tl
              and bool((kf[:, :rank * tl - w] == 0).all()) and torch.equal(kf[:, rank * tl - w:], kc))
    return rank, ok or f"shapes {tuple(kc.shape)} / {tuple(kf.shape)}, key_offset {compact.key_offset}"


def test_context_parallel_view_holds_only_halo_and_local_rows():
    res = _run(_cp_compact)
    for r in res:
        assert r[1] is True, r


# ------------------------------------------------------------------ PP
def _pp(rank, ws):
    from saint_llm_b200.parallel.pipeline import PipelineStage, default_lm_loss, run_1f1b, sync_tied_embedding

    full = _model()
    pp = copy.deepcopy(full)
    torch.manual_seed(9)
    micro = [_ids(1, 16, vocab=full.cfg.vocab_size) for _ in range(4)]
    ref_losses = []
    for ids in micro:
        h, _ = full.backbone(ids)
        loss = default_lm_loss(full, h, ids)
        (loss / len(micro)).backward()
        ref_losses.append(loss.detach())
    stage = PipelineStage(pp)
    out = run_1f1b(stage, micro)
    sync_tied_embedding(stage)
    ok = []
    if stage.last:
        ok.append(_close(out, torch.stack(ref_losses).mean(), 1e-5))
    fp = dict(full.named_parameters())
    own = [f"blocks.{i}." for i in range(stage.lo, stage.hi)]
    for n, p in pp.named_parameters():
        mine = any(n.startswith(o) for o in own) or (n.startswith("embed.") and (stage.first or stage.last)) or \
            (n.startswith("final_norm.") and stage.last)
        if mine and fp[n].grad is not None:
            ok.append(_close(p.grad, fp[n].grad))
    return rank, all(ok), len(ok)


def test_pipeline_1f1b_two_stages():
    res = _run(_pp)
    for r in res:
        assert r[1] is True and r[2] > 5, r


def _pp_cp(rank, ws):
    """Config 4's layout in miniature: 2 pipeline stages x 2 context-parallel ranks each."""
    from saint_llm_b200.parallel.pipeline import (PipelineStage, default_lm_loss, run_1f1b, sync_cp_grads,
                                                  sync_tied_embedding)

    cp_n = 2
    cp_groups = [dist.new_group([s * cp_n + c for c in range(cp_n)]) for s in range(ws // cp_n)]
    pp_groups = [dist.new_group([s * cp_n + c for s in range(ws // cp_n)]) for c in range(cp_n)]
    full = _model()
    pp = copy.deepcopy(full)
    torch.manual_seed(9)
    micro = [_ids(1, 32, vocab=full.cfg.vocab_size) for _ in range(3)]
    ref_losses = []
    for ids in micro:
        h, _ = full.backbone(ids)
        loss = default_lm_loss(full, h, ids)
        (loss / len(micro)).backward()
        ref_losses.append(loss.detach())
    stage = PipelineStage(pp, pp_groups[rank % cp_n], cp_group=cp_groups[rank // cp_n])
    out = run_1f1b(stage, micro)
    sync_cp_grads(stage)
    sync_tied_embedding(stage)
    ok = []
    if stage.last:
        tot = out.detach().clone()
        dist.all_reduce(tot, group=stage.cp_group)
        ok.append(_close(tot, torch.stack(ref_losses).mean(), 1e-5))
    fp = dict(full.named_parameters())
    own = [f"blocks.{i}." for i in range(stage.lo, stage.hi)]
    for n, p in pp.named_parameters():
        mine = any(n.startswith(o) for o in own) or (n.startswith("embed.") and (stage.first or stage.last)) or \
            (n.startswith("final_norm.") and stage.last)
        if mine and fp[n].grad is not None:
            ok.append(_close(p.grad, fp[n].grad))
    return rank, all(ok), len(ok)


def test_pipeline_with_context_parallel_stages():
    """PP=2 x CP=2 on 4 gloo ranks: each stage's sequence split over its CP pair, 1F1B between
    the stages; losses and every owned gradient equal one process."""
    res = _run(_pp_cp, ws=4)
    for r in res:
        assert r[1] is True and r[2] > 5, r


# ------------------------------------------------------------------ DualPipe-V
def test_dualpipe_schedule_is_valid():
    from saint_llm_b200.parallel.dualpipe import build_schedule, owner

    for P, M in [(1, 3), (2, 1), (2, 4), (3, 6), (4, 8), (4, 3)]:
        ticks = build_schedule(P, M)
        when = {}
        for t, row in enumerate(ticks):
            for r, op in enumerate(row):
                if op is not None:
                    assert owner(op.v, P) == r
                    assert (op.kind, op.v, op.i) not in when
                    when[(op.kind, op.v, op.i)] = t
        S = 2 * P
        assert len(when) == 2 * S * M
        for (kind, v, i), t in when.items():
            if kind == "F" and v > 0:
                assert when[("F", v - 1, i)] < t
            if kind == "B":
                assert when[("F", v, i)] < t
                if v < S - 1:
                    assert when[("B", v + 1, i)] < t
        # the V overlaps the two chunks: fewer ticks than running the 2P stages one after another
        assert len(ticks) < 2 * S * M or M == 1 or P == 1


def _dualpipe(rank, ws):
    from saint_llm_b200.parallel.dualpipe import DualPipeV, run_dualpipe
    from saint_llm_b200.parallel.pipeline import default_lm_loss

    full = _model()
    pp = copy.deepcopy(full)
    torch.manual_seed(9)
    micro = [_ids(1, 16, vocab=full.cfg.vocab_size) for _ in range(5)]
    ref_losses = []
    for ids in micro:
        h, _ = full.backbone(ids)
        loss = default_lm_loss(full, h, ids)
        (loss / len(micro)).backward()
        ref_losses.append(loss.detach())
    pipe = DualPipeV(pp)
    out = run_dualpipe(pipe, micro)
    ok = []
    if rank == 0:
        ok.append(_close(out, torch.stack(ref_losses).mean(), 1e-5))
    fp = dict(full.named_parameters())
    own = [f"blocks.{i}." for lo, hi in pipe.bounds.values() for i in range(lo, hi)]
    for n, p in pp.named_parameters():
        mine = any(n.startswith(o) for o in own) or (rank == 0 and n.startswith(("embed.", "final_norm.")))
        if mine and fp[n].grad is not None:
            ok.append(p.grad is not None and _close(p.grad, fp[n].grad))
    return rank, all(ok), len(ok)


def _dualpipe_cp(rank, ws):
    """DualPipe-V over 2 pipeline ranks, each chunk's sequence split over a CP pair."""
    from saint_llm_b200.parallel.dualpipe import DualPipeV, run_dualpipe
    from saint_llm_b200.parallel.pipeline import default_lm_loss, sync_cp_grads

    cp_n = 2
    cp_groups = [dist.new_group([s * cp_n + c for c in range(cp_n)]) for s in range(ws // cp_n)]
    pp_groups = [dist.new_group([s * cp_n + c for s in range(ws // cp_n)]) for c in range(cp_n)]
    full = _model()
    pp = copy.deepcopy(full)
    torch.manual_seed(9)
    micro = [_ids(1, 32, vocab=full.cfg.vocab_size) for _ in range(4)]
    micro[1][:, 20:22] = full.cfg.tokenizer_slots.image_pad
    ref_losses = []
    for ids in micro:
        h, _ = full.backbone(ids)
        loss = default_lm_loss(full, h, ids)
        (loss / len(micro)).backward()
        ref_losses.append(loss.detach())
    pipe = DualPipeV(pp, pp_groups[rank % cp_n], cp_group=cp_groups[rank // cp_n])
    out = run_dualpipe(pipe, micro)
    sync_cp_grads(pipe)
    ok = []
    if pipe.rank == 0:
        tot = out.detach().clone()
        dist.all_reduce(tot, group=pipe.cp_group)
        ok.append(_close(tot, torch.stack(ref_losses).mean(), 1e-5))
    fp = dict(full.named_parameters())
    own = [f"blocks.{i}." for lo, hi in pipe.bounds.values() for i in range(lo, hi)]
    for n, p in pp.named_parameters():
        mine = any(n.startswith(o) for o in own) or (pipe.rank == 0 and n.startswith(("embed.", "final_norm.")))
        if mine and fp[n].grad is not None:
            ok.append(p.grad is not None and _close(p.grad, fp[n].grad))
    return rank, all(ok), len(ok)


def test_dualpipe_v_with_context_parallel_chunks():
    """DualPipe-V (2 pipeline ranks) x CP=2 on 4 gloo ranks equals one process."""
    res = _run(_dualpipe_cp, ws=4)
    for r in res:
        assert r[1] is True and r[2] > 5, r


@pytest.mark.parametrize("ws", [2, 4])
def test_dualpipe_v_matches_single_process(ws):
    res = _run(_dualpipe, ws)
    for r in res:
        assert r[1] is True and r[2] >= 3, r


class _OneWork:
    """The whole group's transfers behind one handle, as NCCL returns them."""

    def __init__(self, works):
        self.works = works

    def wait(self):
        for w in self.works:
            w.wait()
        return True


def _dualpipe_coalesced(rank, ws):
    """DualPipe-V when the backend returns one work for a tick's whole group of transfers
    (NCCL's coalescing), emulated over gloo by wrapping the per-op works."""
    import saint_llm_b200.parallel.dualpipe as dp

    real = dist.batch_isend_irecv
    dp.dist.batch_isend_irecv = lambda ops: [_OneWork(real(ops))]
    try:
        return _dualpipe(rank, ws)
    finally:
        dp.dist.batch_isend_irecv = real


def test_dualpipe_v_with_coalesced_group_works():
    res = _run(_dualpipe_coalesced, 2)
    for r in res:
        assert r[1] is True and r[2] >= 3, r


# ------------------------------------------------------------------ the same on GPUs over NCCL
_two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


@pytest.mark.gpu
@_two_gpus
@pytest.mark.parametrize("name", ["tp", "cp", "pp", "dualpipe"])
def test_parallel_layouts_on_gpus_over_nccl(name):
    """TP, CP, 1F1B and DualPipe-V with NCCL collectives and p2p between two GPUs, checked
    against the same model run in one process (NCCL_NVLS_ENABLE=0 as for every multi-GPU test)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    fn = {"tp": _tp, "cp": _cp, "pp": _pp, "dualpipe": _dualpipe}[name]
    res = _run(fn, 2, nccl=True)
    for r in res:
        assert r[1] is True, r


_four_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4,
                                reason="needs 4 GPUs")


@pytest.mark.gpu
@_four_gpus
@pytest.mark.parametrize("name", ["pp_cp", "dualpipe_cp"])
def test_pipeline_with_context_parallel_on_four_gpus(name):
    """Config 4's PP x CP layout (2 pipeline ranks x CP=2) over NCCL on four GPUs against one
    process (NVLS off)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    fn = {"pp_cp": _pp_cp, "dualpipe_cp": _dualpipe_cp}[name]
    res = _run(fn, 4, nccl=True)
    for r in res:
        assert r[1] is True, r


def _pp_cp_job(rank, ws):
    """``build_training`` with RunConfig(pp=2, cp=2) on 4 ranks (1F1B, then DualPipe-V): one
    step equals one process stepping on the main + MTP loss of the same micro-batches."""
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.optim import MuonAdamW, split_for_muon_adamw
    from saint_llm_b200.train.launch import build_training
    from saint_llm_b200.train.losses import make_loss_fn

    cfg = ModelConfig.tiny()
    cfg = cfg.model_copy(update={"moe": cfg.moe.model_copy(update={"sequence_balance_weight": 0.5})})
    torch.manual_seed(4)
    batch = torch.randint(0, cfg.vocab_size, (2, 1, 32))
    torch.manual_seed(0)
    ref = SaintLLM(cfg)
    opt = MuonAdamW(*split_for_muon_adamw(ref), lr=0.02, adamw_lr=3e-3, qk_clip_enabled=False)
    loss_fn = make_loss_fn(cfg.mtp, moe_cfg=cfg.moe, fused=False)
    want = 0.0  # the reported value: main + MTP (the balance term only enters the gradients)
    for i in range(2):
        loss = loss_fn(ref, batch[i]) / 2
        loss.backward()
        want += float(loss.detach()) - cfg.moe.sequence_balance_weight * float(ref.aux_loss().detach()) / 2
    ref_grads = {n: p.grad.clone() for n, p in ref.named_parameters() if p.grad is not None}
    init = {n: p.detach().clone() for n, p in ref.named_parameters()}
    opt.step()
    refp = dict(ref.named_parameters())
    out = []
    for schedule in ("1f1b", "dualpipe"):
        run = RunConfig(pp=2, cp=2, pp_schedule=schedule, grad_accum=2, micro_batch=1, seq_len=32, lr=0.02,
                        adamw_lr=3e-3, seed=0, param_dtype="float32", compute_dtype="float32")
        job = build_training(cfg, run, DEV, qk_clip=False)
        grads: dict = {}
        real_step = job.optimizer.step

        def step_and_record(*a, _g=grads, _m=job.model, _s=real_step, **k):  # the synchronised gradients
            _g.update({n: p.grad.detach().cpu() for n, p in _m.named_parameters() if p.grad is not None})
            return _s(*a, **k)

        job.optimizer.step = step_and_record
        got = job.step(batch)
        # the weights this rank updated (its blocks, and the ends it holds) match; the rest
        # of its model copy is untouched
        mine = [f"blocks.{i}." for i in range(len(job.model.blocks)) if hasattr(job.model.blocks[i], "attention")]
        first = job.step.stage.first if schedule == "1f1b" else job.step.stage.rank == 0
        last = job.step.stage.last if schedule == "1f1b" else job.step.stage.rank == 0
        owned = [n for n, _ in job.model.named_parameters()
                 if any(n.startswith(o) for o in mine) or (n.startswith("embed.") and (first or last))
                 or (n.startswith(("final_norm.", "mtp.")) and last)]
        cur = {n: p.detach().cpu() for n, p in job.model.named_parameters()}
        # gradients: exact up to summation order (floor: cancelling sums such as the mHC biases')
        g_worst = max(float((grads[n] - ref_grads[n]).abs().max() / ref_grads[n].abs().max().clamp(min=1e-5))
                      for n in owned if n in ref_grads)
        # weights: Newton-Schulz amplifies that noise for experts that saw few tokens (low-rank
        # gradients); a wrong reduction or a missed update would be off by the whole move
        w_ok = all(float((cur[n].detach() - refp[n].detach()).abs().max())
                   <= 5e-2 * float((refp[n].detach() - init[n]).abs().max()) + 2e-5 for n in owned)
        n_blocks = sum(1 for b in job.model.blocks if hasattr(b, "attention"))
        # a checkpoint of the pipeline job holds the whole model; a job built with other
        # weights loads its own stage back from it
        path = os.path.join(os.environ["SV4_TEST_CKPT_DIR"], schedule)
        job.save(path, step=1)
        from saint_llm_b200.train.checkpoint import load_sharded

        saved = load_sharded(path, rank=rank)["model"]
        other = build_training(cfg, run.model_copy(update={"seed": 7}), DEV, qk_clip=False)
        other.load(path)
        theirs = {n: p.detach().cpu() for n, p in other.model.named_parameters()}
        same = all(torch.equal(theirs[n].detach(), cur[n].detach()) for n in owned)
        ckpt_ok = set(saved) == set(ref.state_dict()) and same
        out.append((abs(got - want) < 1e-5, g_worst < 1e-3 and w_ok and set(grads) <= set(ref_grads) and ckpt_ok,
                    n_blocks))
    return rank, out


def test_build_training_pipeline_and_context_parallel(tmp_path):
    os.environ["SV4_TEST_CKPT_DIR"] = str(tmp_path)  # inherited by the spawned ranks
    res = _run(_pp_cp_job, ws=4)
    for r in res:
        assert isinstance(r[1], list), r
        for ok_loss, ok_weights, n_blocks in r[1]:
            assert ok_loss and ok_weights and n_blocks == 2, r


def _cp_job(rank, ws):
    from saint_llm_b200.config import ModelConfig, RunConfig
    from saint_llm_b200.train.launch import build_training

    cfg = ModelConfig.tiny()
    run = RunConfig(cp=ws, grad_accum=2, micro_batch=1, seq_len=32, lr=0.02, adamw_lr=3e-3,
                    param_dtype="float32", compute_dtype="float32")
    job = build_training(cfg, run, DEV)
    torch.manual_seed(4)
    batch = torch.randint(0, cfg.vocab_size, (2, 1, 32))
    return rank, [job.step(batch) for _ in range(3)]


def test_build_training_context_parallel_only():
    """RunConfig(cp=2) alone (one pipeline stage, MuonClip on): both ranks report the same
    decreasing losses."""
    res = _run(_cp_job, ws=2)
    assert all(isinstance(r[1], list) for r in res), res
    a, b = res[0][1], res[1][1]
    assert all(abs(x - y) < 1e-6 for x, y in zip(a, b, strict=True)) and a[-1] < a[0], res


@pytest.mark.gpu
@_four_gpus
def test_build_training_pipeline_and_context_parallel_on_four_gpus(tmp_path):
    """The builder-level PP=2 x CP=2 check with NCCL on four GPUs (the model math on the eager
    fp32 path, compared with one CPU process; NVLS off)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["SV4_TEST_CKPT_DIR"] = str(tmp_path)
    res = _run(_pp_cp_job, 4, nccl=True)
    for r in res:
        assert isinstance(r[1], list), r
        for ok_loss, ok_weights, n_blocks in r[1]:
            assert ok_loss and ok_weights and n_blocks == 2, r

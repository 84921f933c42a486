"""Fused MoE layer on the native kernels (local experts; the EP wrapper is parallel.ep).

Forward of ``DeepSeekMoE`` on CUDA::

    h      = RMSNorm(x)                                    (native)
    idx, g = router(h)                                     (learned or hash)
    plan   = moe_route_plan(idx)                           expert segments padded to 128 rows,
                                                           slot positions, row->token map (device)
    x_p    = gather(h, plan)                               (M_pad, D)
    act    = grouped GEMM [W_gate | W_up] + SwiGLU epilogue (M_pad, I)   (+ pre-acts saved)
    y      = grouped GEMM W_down                           (M_pad, D)
    out    = combine(y, plan, g) + sum_s SwiGLU_s(h)       shared experts: dense fused SwiGLU

Backward reverses each step; weight gradients go straight into ``main_grad`` (fp32)
through the accumulate epilogue of the grouped wgrad GEMMs.  No host synchronisation:
problem tables for the grouped GEMMs are built on the device from the routing counts.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from saint_llm_b200.ops import backend, gemm
from saint_llm_b200.ops.linear import accumulate_weight_grad

_PROB_INTS: int | None = None


def _prob_table(n: int, device: torch.device) -> Tensor:
    global _PROB_INTS
    if _PROB_INTS is None:
        _PROB_INTS = backend.ext().problem_bytes() // 4
    return torch.empty(n, _PROB_INTS, dtype=torch.int32, device=device)


def _bf16c(t: Tensor) -> Tensor:
    return (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)).contiguous()


class RoutePlan:
    """Device-side routing layout for one MoE call."""

    def __init__(self, idx: Tensor, n_experts: int, k: int) -> None:
        ext = backend.ext()
        dev = idx.device
        n_pairs = idx.numel()
        self.n_experts = n_experts
        self.k = k
        self.m_cap = n_pairs + n_experts * 128
        self.counts = torch.empty(n_experts, dtype=torch.int32, device=dev)
        self.seg_start = torch.empty(n_experts, dtype=torch.int32, device=dev)
        self.seg_rows = torch.empty(n_experts, dtype=torch.int32, device=dev)
        self.total = torch.empty(1, dtype=torch.int32, device=dev)
        self.pos = torch.empty(idx.shape[0], k, dtype=torch.int32, device=dev)
        self.row_token = torch.full((self.m_cap,), -1, dtype=torch.int32, device=dev)
        ext.moe_route_plan(idx.reshape(-1).to(torch.int64).contiguous(), n_experts, k, self.counts, self.seg_start,
                           self.seg_rows, self.total, self.pos, self.row_token, gemm.error_word(dev))

    def row_pair(self) -> Tensor:
        """(m_cap,) int32: the (token, slot) pair index t * k + j of each expert row, -1 for
        padding rows."""
        rp = torch.full((self.m_cap,), -1, dtype=torch.int32, device=self.pos.device)
        n = self.pos.numel()
        rp.index_put_((self.pos.reshape(-1).long(),), torch.arange(n, dtype=torch.int32, device=rp.device))
        return rp

    def problems(self, mode: int, D: int, I: int) -> tuple[Tensor, Tensor, int]:
        n = self.n_experts * (2 if mode == 4 else 1)
        probs = _prob_table(n, self.pos.device)
        total = torch.empty(1, dtype=torch.int32, device=self.pos.device)
        backend.ext().build_moe_problems(self.seg_start, self.seg_rows, mode, D, I, probs, total)
        return probs, total, n


_EMPTY: dict[torch.device, Tensor] = {}


def _empty(dev: torch.device) -> Tensor:
    t = _EMPTY.get(dev)
    if t is None:
        t = torch.empty(0, device=dev)
        _EMPTY[dev] = t
    return t


def fp8_expert_weights(pool: nn.Module) -> tuple:
    """Block-scaled FP8 gate/up (interleaved 64-row groups) and down weights of a routed
    expert pool: cached on the pool when ``pool.fp8_weight_cache`` says so ("always", or
    "auto" for a pool sharded by expert parallelism, whose FP8 copy is small), otherwise
    quantised for this call only (a whole unsharded pool's FP8 copy, 15.5 GB for config 3,
    does not fit on one GPU next to its bf16 weights, fp32 gradients and Muon state)."""
    from saint_llm_b200.ops import fp8

    policy = getattr(pool, "fp8_weight_cache", "auto")
    sharded = getattr(pool, "n_global_experts", pool.n_experts) > pool.n_experts
    wg, wu, wd = pool.gate_weight, pool.up_weight, pool.down_weight
    if policy == "always" or (policy == "auto" and sharded):
        return (fp8.cached_weight(pool, "_fp8_gu", [wg, wu], "gu"),
                fp8.cached_weight(pool, "_fp8_down", [wd], "rows"))
    return fp8.transient_weight([wg, wu], "gu"), fp8.transient_weight([wd], "rows")


def fp8_swiglu_experts(xq, gu, down, plan, D: int, I: int, clamps, err,
                       y_out: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """FP8 forward of a grouped SwiGLU expert pool over quantised rows ``xq`` laid out by
    ``plan`` (``RoutePlan`` or an owner-side segment plan).  Returns (act, pre, y): the
    bf16 SwiGLU output and pre-activations [gate | up] (saved for the bf16 backward) and the
    down projection (written into ``y_out`` when given: contiguous, one row per row of xq)."""
    from saint_llm_b200.ops import fp8

    ext = backend.ext()
    rows = xq.q.shape[0]
    dev = xq.q.device
    gmax, lo, hi = clamps
    act = torch.empty(rows, I, dtype=torch.bfloat16, device=dev)
    pre = torch.empty(rows, 2 * I, dtype=torch.bfloat16, device=dev)
    pr, tot, n = plan.problems(6, D, I)
    ext.grouped_gemm_fp8(0, xq.q, xq.sf, gu.q, gu.sf, act, pre, pr, tot, n, 2 * I, gmax, lo, hi, err)
    aq = fp8.quantize_rows(act)
    y = torch.empty(rows, D, dtype=torch.bfloat16, device=dev) if y_out is None else y_out
    pr, tot, n = plan.problems(7, D, I)
    ext.grouped_gemm_fp8(1, aq.q, aq.sf, down.q, down.sf, y, None, pr, tot, n, D, 0.0, 0.0, 0.0, err)
    return act, pre, y


def fp8_pool_ok(pool: nn.Module) -> bool:
    """The pool trains with the block-scaled FP8 forward (``linear_quant == "fp8"``, CUDA
    shapes that fit the FP8 GEMM: I and D multiples of 128)."""
    if getattr(pool, "linear_quant", "bf16") != "fp8":
        return False
    _, i, d = pool.gate_weight.shape
    return i % 128 == 0 and d % 128 == 0


class _RoutedExpertsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor, idx: Tensor, gate: Tensor, wg: Tensor, wu: Tensor, wd: Tensor,  # type: ignore[override]
                clamps: tuple[float, float, float], pool: nn.Module | None = None) -> Tensor:
        ext = backend.ext()
        dev = h.device
        T, D = h.shape
        E, I, _ = wg.shape
        k = idx.shape[1]
        gmax, lo, hi = clamps
        err = gemm.error_word(dev)
        plan = RoutePlan(idx, E, k)
        hb = _bf16c(h)
        if pool is not None:  # block-scaled FP8 forward, bf16 straight-through backward
            from saint_llm_b200.ops import fp8

            gu, down = fp8_expert_weights(pool)
            xq = fp8.gather_quantize_rows(hb, plan.row_token, plan.m_cap)
            act, pre, y = fp8_swiglu_experts(xq, gu, down, plan, D, I, clamps, err)
            del xq, gu, down
        else:
            x_p = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
            ext.moe_gather(hb, plan.row_token, x_p, err)
            wgb, wub, wdb = _bf16c(wg), _bf16c(wu), _bf16c(wd)
            act = torch.empty(plan.m_cap, I, dtype=torch.bfloat16, device=dev)
            pre = torch.empty(plan.m_cap, 2 * I, dtype=torch.bfloat16, device=dev)
            e0 = _empty(dev)
            pr, tot, n = plan.problems(0, D, I)
            ext.grouped_gemm(0, x_p, wgb, wub, act, pre, e0, pr, tot, n, gmax, lo, hi, 0, False, err)
            y = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
            pr, tot, n = plan.problems(1, D, I)
            ext.grouped_gemm(1, act, wdb, wdb, y, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, False, err)
            del x_p
        del act  # recomputed from pre in the backward (saves rows x I bf16 per layer)
        out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        gf = gate.float().contiguous()
        ext.moe_combine(y, plan.pos, gf, out, err)
        del y  # the gate gradient is recovered in the backward without the expert outputs
        ctx.save_for_backward(hb, gf, pre, wg, wu, wd)
        ctx.plan = plan
        ctx.clamps = clamps
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        hb, gf, pre, wg, wu, wd = ctx.saved_tensors
        plan: RoutePlan = ctx.plan
        ext = backend.ext()
        dev = hb.device
        T, D = hb.shape
        E, I, _ = wg.shape
        gmax, lo, hi = ctx.clamps
        err = gemm.error_word(dev)
        e0 = _empty(dev)
        dy = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
        dgate = torch.zeros_like(gf)
        ext.moe_combine_bwd(_bf16c(dout), None, plan.pos, gf, dy, None, err)
        ext.moe_zero_pad_rows(plan.row_token, dy)
        wgb, wub, wdb = _bf16c(wg), _bf16c(wu), _bf16c(wd)
        # down projection: d_act = dy Wd
        dact = torch.empty(plan.m_cap, I, dtype=torch.bfloat16, device=dev)
        pr, tot, n = plan.problems(2, D, I)
        ext.grouped_gemm(2, dy, wdb, wdb, dact, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, False, err)
        # SwiGLU backward, recomputing the activation from the saved pre-activations; the
        # gate gradient <dout, y> = <dact, act> / gate of each (token, slot) row comes along
        dpre = torch.empty(plan.m_cap, 2 * I, dtype=torch.bfloat16, device=dev)
        act = torch.empty(plan.m_cap, I, dtype=torch.bfloat16, device=dev)
        ext.swiglu_bwd_gate(dact, pre, dpre, gmax, lo, hi, act, plan.row_pair(), gf, dgate, err)
        del dact
        # dWd += dy^T act
        dwd_buf = getattr(wd, "main_grad", None)
        acc_d = dwd_buf is not None
        if dwd_buf is None:
            dwd_buf = torch.zeros(E, D, I, dtype=torch.float32, device=dev)
        pr, tot, n = plan.problems(5, D, I)
        ext.grouped_gemm(4, dy, act, act, dwd_buf, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, True, err)
        del act
        # gate/up: dx_p = dpre [Wg; Wu] ; d[Wg|Wu] += dpre^T x_p
        dxp = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
        pr, tot, n = plan.problems(3, D, I)
        ext.grouped_gemm(3, dpre, wgb, wub, dxp, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, I, False, err)
        x_p = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
        ext.moe_gather(hb, plan.row_token, x_p, err)
        mg_g, mg_u = getattr(wg, "main_grad", None), getattr(wu, "main_grad", None)
        if mg_g is not None and mg_u is not None and mg_u.data_ptr() == mg_g.data_ptr() + mg_g.numel() * 4:
            joint, acc_gu = mg_g, True
        else:
            joint, acc_gu = torch.zeros(2, E, I, D, dtype=torch.float32, device=dev), False
        pr, tot, n = plan.problems(4, D, I)
        ext.grouped_gemm(4, dpre, x_p, x_p, joint, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, True, err)
        dh = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        ext.moe_combine(dxp, plan.pos, None, dh, err)
        dwg = None if acc_gu else joint[0].to(wg.dtype)
        dwu = None if acc_gu else joint[1].to(wu.dtype)
        dwd = None if acc_d else dwd_buf.to(wd.dtype)
        return dh, None, dgate, dwg, dwu, dwd, None, None


class _SharedSwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor, wg: Tensor, wu: Tensor, wd: Tensor, clamps: tuple[float, float, float]):  # type: ignore[override]
        ext = backend.ext()
        dev = h.device
        T, D = h.shape
        I = wg.shape[0]
        hb = _bf16c(h)
        act = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
        pre = torch.empty(T, 2 * I, dtype=torch.bfloat16, device=dev)
        ext.swiglu_dense(hb, _bf16c(wg), _bf16c(wu), act, pre, *clamps, gemm.error_word(dev))
        y = gemm.gemm_nt(act, _bf16c(wd))
        ctx.save_for_backward(hb, pre, wg, wu, wd)  # act is recomputed from pre
        ctx.clamps = clamps
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        hb, pre, wg, wu, wd = ctx.saved_tensors
        ext = backend.ext()
        dev = hb.device
        I = wg.shape[0]
        dyb = _bf16c(dy)
        dact = gemm.gemm_nt(dyb, _bf16c(wd).t())
        dpre = torch.empty_like(pre)
        act = torch.empty(pre.shape[0], I, dtype=torch.bfloat16, device=dev)
        ext.swiglu_bwd(dact, pre, dpre, *ctx.clamps, act)
        dwd = accumulate_weight_grad(wd, dyb, act)
        dh = torch.empty_like(hb)
        ext.swiglu_dense_dgrad(dpre, _bf16c(wg), _bf16c(wu), dh, gemm.error_word(dev))
        dwg = accumulate_weight_grad(wg, dpre[:, :I], hb)
        dwu = accumulate_weight_grad(wu, dpre[:, I:], hb)
        return dh, dwg, dwu, dwd, None


def _cat(ws: list[Tensor], dim: int) -> Tensor:
    # rebuilt on every call: native optimizer kernels update weights in place without
    # bumping torch's version counters, so a cached copy could go stale
    return torch.cat([_bf16c(w.detach()) for w in ws], dim=dim)


class _DensePlan:
    """Problem table of one dense (T-row) SwiGLU / down product for the FP8 grouped GEMM."""

    def __init__(self, rows: int, device: torch.device) -> None:
        self.seg_start = torch.zeros(1, dtype=torch.int32, device=device)
        self.seg_rows = torch.full((1,), rows, dtype=torch.int32, device=device)

    def problems(self, mode: int, D: int, I: int) -> tuple[Tensor, Tensor, int]:
        probs = _prob_table(1, self.seg_start.device)
        total = torch.empty(1, dtype=torch.int32, device=self.seg_start.device)
        backend.ext().build_moe_problems(self.seg_start, self.seg_rows, mode, D, I, probs, total)
        return probs, total, 1


def shared_group_forward(h: Tensor, clamps: tuple[float, float, float], fp8_owner: nn.Module | None,
                         ws: list[Tensor]) -> tuple[Tensor, tuple]:
    """Forward of several shared SwiGLU experts fused into one (see ``_SharedGroupFn``).
    Returns the output and what the backward needs."""
    ext = backend.ext()
    dev = h.device
    n = len(ws) // 3
    wgs, wus, wds = list(ws[:n]), list(ws[n:2 * n]), list(ws[2 * n:])
    T = h.shape[0]
    I = sum(w.shape[0] for w in wgs)
    hb = _bf16c(h)
    if fp8_owner is not None:
        from saint_llm_b200.ops import fp8

        gu = fp8.cached_weight(fp8_owner, "_fp8_shared_gu", wgs + wus, "gu")
        down = fp8.cached_weight(fp8_owner, "_fp8_shared_down", wds, "cols")
        act, pre, y = fp8_swiglu_experts(fp8.quantize_rows(hb), gu, down, _DensePlan(T, dev), hb.shape[1], I,
                                         clamps, gemm.error_word(dev))
    else:
        wg, wu, wd = _cat(wgs, 0), _cat(wus, 0), _cat(wds, 1)
        act = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
        pre = torch.empty(T, 2 * I, dtype=torch.bfloat16, device=dev)
        ext.swiglu_dense(hb, wg, wu, act, pre, *clamps, gemm.error_word(dev))
        y = gemm.gemm_nt(act, wd)
    return y, (hb, pre)  # act is recomputed from pre in the backward


def shared_group_backward(saved: tuple, ws: list[Tensor], clamps: tuple[float, float, float],
                          dy: Tensor) -> tuple[Tensor, list[Tensor | None]]:
    """Backward of ``shared_group_forward``: (dh, weight gradients in ``ws`` order; None
    where they went into ``main_grad``)."""
    hb, pre = saved
    n = len(ws) // 3
    wgs, wus, wds = ws[:n], ws[n:2 * n], ws[2 * n:]
    ext = backend.ext()
    dev = hb.device
    wg, wu, wd = _cat(list(wgs), 0), _cat(list(wus), 0), _cat(list(wds), 1)
    I = wg.shape[0]
    dyb = _bf16c(dy)
    dact = gemm.gemm_nt(dyb, wd.t())
    dpre = torch.empty_like(pre)
    act = torch.empty(pre.shape[0], I, dtype=torch.bfloat16, device=dev)
    ext.swiglu_bwd(dact, pre, dpre, *clamps, act)
    del dact
    dh = torch.empty_like(hb)
    ext.swiglu_dense_dgrad(dpre, wg, wu, dh, gemm.error_word(dev))
    off = 0
    dg, du, dd = [], [], []
    for e in range(n):
        ie = wgs[e].shape[0]
        dg.append(accumulate_weight_grad(wgs[e], dpre[:, off:off + ie], hb))
        du.append(accumulate_weight_grad(wus[e], dpre[:, I + off:I + off + ie], hb))
        dd.append(accumulate_weight_grad(wds[e], dyb, act[:, off:off + ie]))
        off += ie
    return dh, dg + du + dd


class _SharedGroupFn(torch.autograd.Function):
    """Several shared SwiGLU experts as one: sum_e SwiGLU_e(h) = [Wd_1 .. Wd_n] SwiGLU(h;
    [Wg_1; ..; Wg_n], [Wu_1; ..; Wu_n]) because the activation is element-wise, so the
    forward is one fused SwiGLU GEMM (intermediate width sum I_e) and one down GEMM, and the
    backward one dgrad per GEMM (and one add fewer per extra expert in each direction);
    weight gradients still go to each expert's own weights.

    ``fp8_owner`` (the first expert module): the forward runs the block-scaled FP8 GEMMs
    against the joint weights' FP8 copies cached on that module; the backward is bf16."""

    @staticmethod
    def forward(ctx, h: Tensor, clamps: tuple[float, float, float], fp8_owner: nn.Module | None,  # type: ignore[override]
                *ws: Tensor) -> Tensor:
        y, saved = shared_group_forward(h, clamps, fp8_owner, list(ws))
        ctx.save_for_backward(*saved, *ws)
        ctx.clamps = clamps
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        hb, pre, *ws = ctx.saved_tensors
        dh, grads = shared_group_backward((hb, pre), list(ws), ctx.clamps, dy)
        return (dh, None, None, *grads)


def shared_group_args(h: Tensor, experts: nn.ModuleList | list[nn.Module]) -> tuple | None:
    """(clamps, fp8_owner, weights) when the shared experts can run fused as one, else None."""
    ex = list(experts)
    if len(ex) < 2:
        return None
    clamps = {(float(e.clamp_gate_max), float(e.clamp_linear[0]), float(e.clamp_linear[1])) for e in ex}
    if len(clamps) != 1 or any(e.gate_proj.weight.shape[0] % 64 for e in ex):
        return None
    ws = [e.gate_proj.weight for e in ex] + [e.up_proj.weight for e in ex] + [e.down_proj.weight for e in ex]
    fp8_ok = (getattr(ex[0].gate_proj, "use_real_fp8_gemm", False) and h.shape[-1] % 128 == 0
              and all(e.gate_proj.weight.shape[0] % 128 == 0 for e in ex))
    return clamps.pop(), ex[0] if fp8_ok else None, ws


def shared_experts(h: Tensor, experts: nn.ModuleList | list[nn.Module]) -> Tensor | None:
    """Sum of the shared SwiGLU experts on h (T, D); None when there are none."""
    ex = list(experts)
    if not ex:
        return None
    if len(ex) == 1:
        return shared_swiglu(h, ex[0])
    args = shared_group_args(h, ex)
    if args is None:
        out = shared_swiglu(h, ex[0])
        for e in ex[1:]:
            out = out + shared_swiglu(h, e)
        return out
    clamps, owner, ws = args
    return _SharedGroupFn.apply(h, clamps, owner, *ws)


def shared_swiglu(h: Tensor, expert: nn.Module) -> Tensor:
    lin = expert.clamp_linear
    return _SharedSwiGLUFn.apply(h, expert.gate_proj.weight, expert.up_proj.weight, expert.down_proj.weight,
                                 (float(expert.clamp_gate_max), float(lin[0]), float(lin[1])))


def routed_experts(h: Tensor, idx: Tensor, gate: Tensor, experts: nn.Module) -> Tensor:
    """h (T, D); idx / gate (T, k): sum_j gate[t,j] * expert_{idx[t,j]}(h[t]) over the local expert pool
    (block-scaled FP8 forward when the pool's ``linear_quant`` is "fp8")."""
    return _RoutedExpertsFn.apply(h, idx, gate, experts.gate_weight, experts.up_weight, experts.down_weight,
                                  (float(experts.clamp_gate_max), float(experts.clamp_linear[0]),
                                   float(experts.clamp_linear[1])), experts if fp8_pool_ok(experts) else None)


class Fp8ExpertWeights:
    """Block-scaled FP8 copies of a grouped expert pool (inference: built once, reused).

    ``gu``: gate and up weights stacked per expert as (E * 2I, D) with 64-row groups
    alternating gate / up, so one 128-column tile of the grouped GEMM holds 64 gate and
    the matching 64 up columns (the SwiGLU epilogue needs both); each 128 x 128 scale block
    covers one such group pair.  ``down``: (E * D, I) in 128 x 128 blocks."""

    def __init__(self, experts: nn.Module) -> None:
        from saint_llm_b200.ops import fp8

        wg, wu, wd = experts.gate_weight.detach(), experts.up_weight.detach(), experts.down_weight.detach()
        e, i, d = wg.shape
        if i % 64 or d % 128 or i % 128:
            raise ValueError(f"FP8 experts need I % 128 == 0 and D % 128 == 0 (got I={i}, D={d})")
        gu = torch.stack([wg.reshape(e, i // 64, 64, d), wu.reshape(e, i // 64, 64, d)], dim=2).reshape(e * 2 * i, d)
        self.gu = fp8.quantize_blocks(gu.to(torch.bfloat16))
        self.down = fp8.quantize_blocks(wd.reshape(e * d, i).to(torch.bfloat16))
        self.E, self.I, self.D = e, i, d
        self.clamps = (float(experts.clamp_gate_max), float(experts.clamp_linear[0]), float(experts.clamp_linear[1]))


@torch.no_grad()
def routed_experts_fp8(h: Tensor, idx: Tensor, gate: Tensor, w8: Fp8ExpertWeights) -> Tensor:
    """Inference forward of the routed experts on the block-scaled FP8 grouped GEMM:
    gathered rows and SwiGLU activations are quantised in 1 x 128 blocks on the fly."""
    from saint_llm_b200.ops import fp8

    ext = backend.ext()
    dev = h.device
    T, D = h.shape
    k = idx.shape[1]
    E, I = w8.E, w8.I
    err = gemm.error_word(dev)
    plan = RoutePlan(idx, E, k)
    x_p = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
    ext.moe_gather(_bf16c(h), plan.row_token, x_p, err)
    xq = fp8.quantize_rows(x_p)
    act = torch.empty(plan.m_cap, I, dtype=torch.bfloat16, device=dev)
    pr, tot, n = plan.problems(6, D, I)
    gmax, lo, hi = w8.clamps
    ext.grouped_gemm_fp8(0, xq.q, xq.sf, w8.gu.q, w8.gu.sf, act, None, pr, tot, n, 2 * I, gmax, lo, hi, err)
    aq = fp8.quantize_rows(act)
    y = torch.empty(plan.m_cap, D, dtype=torch.bfloat16, device=dev)
    pr, tot, n = plan.problems(7, D, I)
    ext.grouped_gemm_fp8(1, aq.q, aq.sf, w8.down.q, w8.down.sf, y, None, pr, tot, n, D, 0.0, 0.0, 0.0, err)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    ext.moe_combine(y, plan.pos, gate.float().contiguous(), out, err)
    return out


def enable_fp8_experts(model: nn.Module) -> int:
    """Quantise every grouped expert pool of ``model`` to block-scaled FP8 for inference;
    the no-grad CUDA forward then runs the FP8 grouped GEMMs.  Returns the number of pools.
    Call again after the weights change (the copies are not refreshed automatically)."""
    n = 0
    for mod in model.modules():
        ge = getattr(mod, "grouped_experts", None)
        if ge is not None and hasattr(ge, "gate_weight"):
            ge._fp8_weights = Fp8ExpertWeights(ge)
            n += 1
    return n


def moe_forward(layer: nn.Module, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
    """CUDA forward of ``DeepSeekMoE``."""
    if getattr(layer, "ep_size", 1) > 1:
        from saint_llm_b200.parallel import ep

        return ep.moe_forward_ep(layer, x, token_ids, is_visual)
    if layer.grouped_experts is None or getattr(layer.grouped_experts, "linear_quant", "bf16") == "fp4":
        return _moe_per_module(layer, x, token_ids, is_visual)
    b, t, d = x.shape
    h = layer.norm(x)
    idx, gate, aux = layer.route(h, token_ids, is_visual)
    layer._last_aux_loss = aux
    k = layer.cfg.experts_per_token
    h2 = h.reshape(b * t, d)
    w8 = getattr(layer.grouped_experts, "_fp8_weights", None)
    if w8 is not None and not torch.is_grad_enabled():
        out = routed_experts_fp8(h2, idx.reshape(b * t, k), gate.reshape(b * t, k), w8)
    else:
        out = routed_experts(h2, idx.reshape(b * t, k), gate.reshape(b * t, k), layer.grouped_experts)
    sh = shared_experts(h2, layer.shared_experts)
    if sh is not None:
        out = out + sh
    return out.view(b, t, d)


def _moe_per_module(layer: nn.Module, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
    """Per-module expert layout on CUDA: the routed loop runs on native linears."""
    h = layer.norm(x)
    b, t, d = h.shape
    idx, gate, aux = layer.route(h, token_ids, is_visual)
    layer._last_aux_loss = aux
    k = layer.cfg.experts_per_token
    fh, fi, fg = h.reshape(b * t, d), idx.reshape(b * t, k), gate.reshape(b * t, k)
    routed = torch.zeros_like(fh)
    if layer.grouped_experts is not None:
        routed = layer.grouped_experts(fh, fi, fg)
    else:
        for e, expert in enumerate(layer.routed_experts):
            tok, slot = (fi == e).nonzero(as_tuple=True)
            if tok.numel():
                routed = routed.index_add(0, tok, expert(fh[tok]) * fg[tok, slot].unsqueeze(-1).to(fh.dtype))
    out = routed
    for expert in layer.shared_experts:
        out = out + expert(fh)
    return out.view(b, t, d)


__all__ = ["Fp8ExpertWeights", "RoutePlan", "enable_fp8_experts", "moe_forward", "routed_experts",
           "routed_experts_fp8", "shared_experts", "shared_swiglu"]

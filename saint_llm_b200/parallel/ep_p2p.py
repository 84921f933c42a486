"""Expert parallelism over NVLink peer memory: the dispatch and the combine run inside
this framework's own kernels (``csrc/ep.cu``) as P2P stores and loads into symmetric
buffers, with the routing counts exchanged on the device (no host synchronisation and
no NCCL on the MoE path).  The NCCL all-to-all path in ``parallel.ep`` is the baseline.

Per MoE layer and micro-batch, on every rank (reference behaviour:
``distributed/expert_parallel.py:47-276``, which moves the same rows with two host-synced
``all_to_all_single`` calls per direction)::

    counts  = per-expert pair counts of this rank            (moe_route_plan)
    ep_post_counts -> ep_plan                                 all ranks' counts -> receive layout + gpos
    ep_dispatch    -> ep_signal(X)                            token rows -> owners' receive buffers
    ep_wait_zero(X)                                           owner: all rows arrived; zero padding
    grouped GEMMs (SwiGLU, down) on the receive buffer        owner, local tensor cores
    ep_signal(Y) -> ep_combine                                pull + gate-weighted reduction

and the backward pushes ``gate * dout`` to the owners (``ep_combine_bwd``), runs the
expert backward there and pulls the input gradients back (``ep_dispatch_bwd``).

Buffers (all ranks allocate the same sizes collectively; mapped into every peer by CUDA
IPC): a flag table, a two-slot count table and four buffers shared by every MoE layer --
the receive buffer and the buffers of the expert outputs, the output gradients and the
input gradients.  Capacity ``C`` rows per rank: ``min(ws, capacity_factor) * T * k`` plus
128 rows of padding per local expert.  With the default factor (``ws``) no routing can
overflow: an untrained router can send most tokens to a few ranks.  The owner reads its
received row count once per layer (one host synchronisation) and keeps a right-sized copy of
the received rows as the saved input of the expert weight gradients; the expert
activations are sized the same way, so memory follows the actual routing, not the worst
case.  A smaller factor saves the shared buffers' memory; an overflow is reported as a
native kernel error (never silently dropped).

Reuse of the shared buffers across layers is safe by stream order: a rank dispatches
layer L+1 only after its combine of layer L, which waited for every owner's "outputs
ready" flag; an owner writes outputs of L+1 only after all sources' rows of L+1 arrived.
The backward follows the same argument with the roles swapped.  Between micro-batches a
rank's next forward starts after its own backward, whose last pull waited for every
owner's final expert backward.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor, nn

from saint_llm_b200.ops import backend, gemm
from saint_llm_b200.ops.moe_native import RoutePlan, _bf16c, _empty, _prob_table
from saint_llm_b200.utils.profiling import phase as _phase

PH_CNT, PH_X, PH_Y, PH_DY, PH_DX = 0, 1, 2, 3, 4
MAX_RANKS = 8
FLAG_INTS = 8 * MAX_RANKS


@dataclass
class SymmetricBuffer:
    """A buffer that exists on every rank; ``ptrs[r]`` is rank r's copy in this process's
    address space (``local`` is this rank's own copy)."""

    local: Tensor
    ptrs: list[int]

    def view(self, dtype: torch.dtype, *shape: int) -> Tensor:
        n = 1
        for s in shape:
            n *= s
        return self.local[:n * torch.empty((), dtype=dtype).element_size()].view(dtype).view(*shape)


class SymmetricHeap:
    """Collective allocator over a process group (one rank per GPU).  Every rank must call
    ``alloc`` with the same sizes in the same order."""

    def __init__(self, group: dist.ProcessGroup | None, device: torch.device) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.ws = dist.get_world_size(group)
        if self.ws > MAX_RANKS:
            raise ValueError(f"peer-memory expert parallelism supports up to {MAX_RANKS} ranks (one node)")
        self.device = device
        self._opened: list[int] = []
        self._owned: list[int] = []
        self.bytes = 0
        self.closed = False

    def alloc(self, nbytes: int) -> SymmetricBuffer:
        nbytes = (nbytes + 255) // 256 * 256
        ext = backend.ext()
        if self.closed:
            raise RuntimeError("symmetric heap is closed")
        t, h = ext.symm_alloc(nbytes, self.device.index)
        self._owned.append(t.data_ptr())
        handles: list = [None] * self.ws
        dist.all_gather_object(handles, h, group=self.group)
        ptrs = []
        for r, hr in enumerate(handles):
            if r == self.rank:
                ptrs.append(t.data_ptr())
            else:
                p = ext.symm_open(hr, self.device.index)
                self._opened.append(p)
                ptrs.append(p)
        self.bytes += nbytes
        return SymmetricBuffer(t, ptrs)

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's, after every rank's
        device has finished all work that touches them.  Tensors handed out by ``alloc``
        must not be used afterwards."""
        if self.closed:
            return
        ext = backend.ext()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every peer is done with our memory
        for p in self._opened:
            ext.symm_close(p, self.device.index)
        self._opened.clear()
        dist.barrier(group=self.group)  # every peer has unmapped our memory
        for p in self._owned:
            ext.symm_free(p, self.device.index)
        self._owned.clear()
        self.closed = True


class EmulatedHeap:
    """Single-process stand-in for ``SymmetricHeap``: ``n_ranks`` emulated ranks on one
    device whose "peer" pointers are the other emulated ranks' tensors.  Every emulated
    rank allocates in the same order, exactly as real ranks do."""

    def __init__(self, rank: int, shared: dict) -> None:
        self.rank, self.ws = rank, shared["n"]
        self.device = shared["device"]
        self._shared = shared
        self._count = 0
        self.bytes = 0

    @classmethod
    def create(cls, n_ranks: int, device: torch.device) -> list[EmulatedHeap]:
        shared = {"n": n_ranks, "device": device, "bufs": []}
        return [cls(r, shared) for r in range(n_ranks)]

    def alloc(self, nbytes: int) -> SymmetricBuffer:
        nbytes = (nbytes + 255) // 256 * 256
        bufs = self._shared["bufs"]
        if self._count == len(bufs):
            bufs.append([torch.zeros(nbytes, dtype=torch.uint8, device=self.device) for _ in range(self.ws)])
        copies = bufs[self._count]
        self._count += 1
        self.bytes += nbytes
        return SymmetricBuffer(copies[self.rank], [t.data_ptr() for t in copies])

    def close(self) -> None:
        pass


class P2PExpertComm:
    """Peer-memory buffers and epochs of one expert-parallel group (shared by every MoE
    layer of a model)."""

    def __init__(self, heap: SymmetricHeap | EmulatedHeap, *, n_experts: int, hidden: int, top_k: int,
                 capacity_factor: float | None = None, timeout_s: float = 30.0) -> None:
        self.heap = heap
        self.rank, self.ws = heap.rank, heap.ws
        if n_experts % self.ws:
            raise ValueError(f"{n_experts} experts not divisible by {self.ws} ranks")
        self.E, self.D, self.k = n_experts, hidden, top_k
        self.E_loc = n_experts // self.ws
        self.capacity_factor = float(self.ws if capacity_factor is None else min(capacity_factor, self.ws))
        self.timeout_ns = int(timeout_s * 1e9)
        self.flags = heap.alloc(FLAG_INTS * 4)
        self.cnt = heap.alloc(2 * MAX_RANKS * n_experts * 4)
        self.epoch = [0] * 5
        self.tokens = 0
        self.C = 0
        self.y = self.dy = self.dx = self.xr = None
        self.rows_received = 0  # expert rows this rank owned, summed over calls (host count)
        # side stream for the token traffic that overlaps the shared experts (see moe_forward_p2p)
        dev = heap.device
        self.side = torch.cuda.Stream(dev) if torch.device(dev).type == "cuda" else None

    def next_epoch(self, phase: int) -> int:
        self.epoch[phase] = (self.epoch[phase] + 1) & 0xFFFFFFFF
        return self.epoch[phase]

    def capacity_for(self, tokens: int) -> int:
        c = int(self.capacity_factor * tokens * self.k) + 128 * self.E_loc
        return (c + 127) // 128 * 128

    def ensure(self, tokens: int) -> None:
        """(Re)allocate the row buffers for ``tokens`` tokens per rank (collective)."""
        if tokens <= self.tokens:
            return
        self.tokens = tokens
        self.C = self.capacity_for(tokens)
        row_bytes = self.C * self.D * 2
        self.xr, self.y, self.dy, self.dx = (self.heap.alloc(row_bytes) for _ in range(4))

    def close(self) -> None:
        """Collective release of every buffer (see ``SymmetricHeap.close``)."""
        self.y = self.dy = self.dx = self.xr = None
        self.heap.close()

    def rows(self, buf: SymmetricBuffer) -> Tensor:
        return buf.view(torch.bfloat16, self.C, self.D)


class _SegPlan:
    """Problem tables of the owner-side grouped GEMMs from its receive layout (segments of
    whole 128-row blocks; the padding rows are zero)."""

    def __init__(self, seg_start: Tensor, seg_rows: Tensor) -> None:
        self.seg_start, self.seg_rows = seg_start, seg_rows
        self.n_experts = seg_start.numel()

    def problems(self, mode: int, D: int, I: int) -> tuple[Tensor, Tensor, int]:
        n = self.n_experts * (2 if mode == 4 else 1)
        probs = _prob_table(n, self.seg_start.device)
        total = torch.empty(1, dtype=torch.int32, device=self.seg_start.device)
        backend.ext().build_moe_problems(self.seg_start, self.seg_rows, mode, D, I, probs, total)
        return probs, total, n


class EPCall:
    """One MoE-layer call on one rank, split into the stages between which a rank waits
    for its peers.  The autograd function runs the stages back to back; a single-GPU
    emulation of several ranks runs each stage for every rank before the next one."""

    def __init__(self, comm: P2PExpertComm, layer_key: int, h: Tensor, idx: Tensor, gate: Tensor, wg: Tensor,
                 wu: Tensor, wd: Tensor, clamps: tuple[float, float, float], fp8_pool: nn.Module | None = None) -> None:
        self.comm, self.layer_key, self.clamps = comm, layer_key, clamps
        self.fp8_pool = fp8_pool  # block-scaled FP8 forward of the owner-side experts
        self.hb = _bf16c(h)
        self.T, self.D = h.shape
        self.idx = idx
        self.gf = gate.float().contiguous()
        self.wg, self.wu, self.wd = wg, wu, wd
        self.dev = h.device
        self.err = gemm.error_word(self.dev)
        comm.ensure(self.T)
        # outputs of the dispatch stage, allocated on the caller's stream so they may be
        # written on the side stream and read back on this one after the join
        E_loc, k = wg.shape[0], idx.shape[1]
        self.gpos = torch.empty(self.T, k, dtype=torch.int32, device=self.dev)
        self.seg_start = torch.empty(E_loc, dtype=torch.int32, device=self.dev)
        self.seg_rows = torch.empty(E_loc, dtype=torch.int32, device=self.dev)
        self.seg_pad = torch.empty(E_loc, dtype=torch.int32, device=self.dev)

    # ---------------------------------------------------------------- forward
    def f1_counts(self) -> None:
        c = self.comm
        self.local = RoutePlan(self.idx, c.E, self.idx.shape[1])
        self.e_cnt = c.next_epoch(PH_CNT)
        backend.ext().ep_post_counts(self.local.counts, c.cnt.ptrs, c.flags.ptrs, c.rank, self.e_cnt & 1, self.e_cnt)

    def f2_dispatch(self) -> None:
        c, ext = self.comm, backend.ext()
        idx64 = self.idx.reshape(-1).to(torch.int64).contiguous()
        ext.ep_plan(idx64, self.local.pos, self.local.seg_start, c.cnt.local.view(torch.int32),
                    c.flags.local.view(torch.int32), self.e_cnt & 1, self.e_cnt, c.rank, c.ws, c.C, self.gpos,
                    self.seg_start, self.seg_rows, self.seg_pad, c.timeout_ns, self.err)
        del self.local
        ext.ep_dispatch(self.hb, self.gpos, c.C, c.xr.ptrs, self.err)
        self.e_x = c.next_epoch(PH_X)
        ext.ep_signal(c.flags.ptrs, PH_X, c.rank, self.e_x)

    def f3_experts(self) -> None:
        c, ext = self.comm, backend.ext()
        D, (E_loc, I, _) = self.D, self.wg.shape
        gmax, lo, hi = self.clamps
        xr = c.rows(c.xr)
        ext.ep_wait_zero(c.flags.local.view(torch.int32), PH_X, c.ws, self.e_x, xr, self.seg_start,
                         self.seg_rows, c.timeout_ns, self.err)
        # rows this owner received (expert segments are contiguous and 128-padded): one host
        # read per layer sizes the saved input and the activations by the actual routing
        self.R = int((self.seg_start[-1] + self.seg_pad[-1]).item()) if E_loc else 0
        c.rows_received += self.R
        x_rows = xr[:self.R].clone()
        self.x_saved = x_rows
        plan = _SegPlan(self.seg_start, self.seg_pad)
        if self.fp8_pool is not None:
            from saint_llm_b200.ops import fp8
            from saint_llm_b200.ops.moe_native import fp8_expert_weights, fp8_swiglu_experts

            gu, down = fp8_expert_weights(self.fp8_pool)
            _, self.pre, _ = fp8_swiglu_experts(fp8.quantize_rows(x_rows), gu, down, plan, D, I, self.clamps,
                                                self.err, y_out=c.rows(c.y)[:self.R])
        else:
            e0 = _empty(self.dev)
            act = torch.empty(self.R, I, dtype=torch.bfloat16, device=self.dev)
            self.pre = torch.empty(self.R, 2 * I, dtype=torch.bfloat16, device=self.dev)
            pr, tot, n = plan.problems(0, D, I)
            ext.grouped_gemm(0, x_rows, _bf16c(self.wg), _bf16c(self.wu), act, self.pre, e0, pr, tot, n, gmax,
                             lo, hi, 0, False, self.err)
            wdb = _bf16c(self.wd)
            pr, tot, n = plan.problems(1, D, I)
            ext.grouped_gemm(1, act, wdb, wdb, c.rows(c.y), e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, False,
                             self.err)
            del act  # recomputed from pre in the backward
        self.e_y = c.next_epoch(PH_Y)
        ext.ep_signal(c.flags.ptrs, PH_Y, c.rank, self.e_y)

    def f4_combine(self) -> Tensor:
        c = self.comm
        k = self.idx.shape[1]
        out = torch.empty(self.T, self.D, dtype=torch.bfloat16, device=self.dev)
        self.ypair = torch.empty(self.T * k, self.D, dtype=torch.bfloat16, device=self.dev)
        backend.ext().ep_combine(c.y.ptrs, self.gpos, self.gf, c.C, out, self.ypair, c.flags.local.view(torch.int32),
                                 PH_Y, c.ws, self.e_y, c.timeout_ns, self.err)
        del self.hb
        return out

    # --------------------------------------------------------------- backward
    def b1_push(self, dout: Tensor, dgate: Tensor | None = None) -> None:
        c, ext = self.comm, backend.ext()
        self.dgate = torch.empty_like(self.gf) if dgate is None else dgate
        ext.ep_combine_bwd(_bf16c(dout), self.ypair, self.gf, self.gpos, c.C, c.dy.ptrs, self.dgate, self.err)
        self.ypair.record_stream(torch.cuda.current_stream(self.dev))  # may be a side stream
        del self.ypair
        self.e_dy = c.next_epoch(PH_DY)
        ext.ep_signal(c.flags.ptrs, PH_DY, c.rank, self.e_dy)

    def b2_experts(self) -> None:
        c, ext = self.comm, backend.ext()
        D, (E_loc, I, _) = self.D, self.wg.shape
        gmax, lo, hi = self.clamps
        dev, err = self.dev, self.err
        dy = c.rows(c.dy)
        ext.ep_wait_zero(c.flags.local.view(torch.int32), PH_DY, c.ws, self.e_dy, dy, self.seg_start, self.seg_rows,
                         c.timeout_ns, err)
        plan = _SegPlan(self.seg_start, self.seg_pad)
        e0 = _empty(dev)
        wdb = _bf16c(self.wd)
        dact = torch.empty(self.R, I, dtype=torch.bfloat16, device=dev)
        pr, tot, n = plan.problems(2, D, I)
        ext.grouped_gemm(2, dy, wdb, wdb, dact, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, False, err)
        # SwiGLU backward, recomputing the activation from the saved pre-activations
        dpre = torch.empty(self.R, 2 * I, dtype=torch.bfloat16, device=dev)
        act = torch.empty(self.R, I, dtype=torch.bfloat16, device=dev)
        ext.swiglu_bwd(dact, self.pre, dpre, gmax, lo, hi, act)
        del self.pre, dact
        dwd_buf = getattr(self.wd, "main_grad", None)
        self.acc_d = dwd_buf is not None
        if dwd_buf is None:
            dwd_buf = torch.zeros(E_loc, D, I, dtype=torch.float32, device=dev)
        pr, tot, n = plan.problems(5, D, I)
        ext.grouped_gemm(4, dy, act, act, dwd_buf, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, True, err)
        del act
        pr, tot, n = plan.problems(3, D, I)
        ext.grouped_gemm(3, dpre, _bf16c(self.wg), _bf16c(self.wu), c.rows(c.dx), e0, e0, pr, tot, n, 0.0, 0.0, 0.0,
                         I, False, err)
        x_rows = self.x_saved
        mg_g, mg_u = getattr(self.wg, "main_grad", None), getattr(self.wu, "main_grad", None)
        if mg_g is not None and mg_u is not None and mg_u.data_ptr() == mg_g.data_ptr() + mg_g.numel() * 4:
            joint, self.acc_gu = mg_g, True
        else:
            joint, self.acc_gu = torch.zeros(2, E_loc, I, D, dtype=torch.float32, device=dev), False
        pr, tot, n = plan.problems(4, D, I)
        ext.grouped_gemm(4, dpre, x_rows, x_rows, joint, e0, e0, pr, tot, n, 0.0, 0.0, 0.0, 0, True, err)
        self.joint, self.dwd_buf = joint, dwd_buf
        del self.x_saved
        self.e_dx = c.next_epoch(PH_DX)
        ext.ep_signal(c.flags.ptrs, PH_DX, c.rank, self.e_dx)

    def b3_pull(self) -> tuple[Tensor, Tensor, Tensor | None, Tensor | None, Tensor | None]:
        c = self.comm
        dh = torch.empty(self.T, self.D, dtype=torch.bfloat16, device=self.dev)
        backend.ext().ep_dispatch_bwd(c.dx.ptrs, self.gpos, c.C, dh, c.flags.local.view(torch.int32), PH_DX, c.ws,
                                      self.e_dx, c.timeout_ns, self.err)
        dwg = None if self.acc_gu else self.joint[0].to(self.wg.dtype)
        dwu = None if self.acc_gu else self.joint[1].to(self.wu.dtype)
        dwd = None if self.acc_d else self.dwd_buf.to(self.wd.dtype)
        return dh, self.dgate, dwg, dwu, dwd


FORWARD_STAGES = ("f1_counts", "f2_dispatch", "f3_experts", "f4_combine")


class _P2PExpertsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor, idx: Tensor, gate: Tensor, wg: Tensor, wu: Tensor, wd: Tensor,  # type: ignore[override]
                comm: P2PExpertComm, layer_key: int, clamps: tuple[float, float, float],
                fp8_pool: nn.Module | None = None) -> Tensor:
        call = EPCall(comm, layer_key, h, idx, gate, wg, wu, wd, clamps, fp8_pool)
        with _phase("ep.dispatch"):
            call.f1_counts()
            call.f2_dispatch()
        with _phase("ep.experts_fwd"):
            call.f3_experts()
        ctx.call = call
        with _phase("ep.combine"):
            return call.f4_combine()

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        call: EPCall = ctx.call
        with _phase("ep.combine_bwd"):
            call.b1_push(dout)
        with _phase("ep.experts_bwd"):
            call.b2_experts()
        with _phase("ep.dispatch_bwd"):
            dh, dgate, dwg, dwu, dwd = call.b3_pull()
        del ctx.call
        return dh, None, dgate, dwg, dwu, dwd, None, None, None, None


class _P2PMoEFn(torch.autograd.Function):
    """Routed experts over peer memory plus the fused shared experts, overlapped: the count
    exchange and the token dispatch run on the communicator's side stream while the shared
    experts' GEMMs run on the caller's stream (the dispatch is NVLink-bound, the GEMMs are
    tensor-core-bound); the owner-side experts start after both streams join.  The backward
    pushes the output gradients to the owners on the side stream while the shared experts'
    backward runs.  Every tensor the side stream touches is either allocated on the
    caller's stream before the fork or recorded on the side stream before it is freed."""

    @staticmethod
    def forward(ctx, h: Tensor, idx: Tensor, gate: Tensor, comm: P2PExpertComm, layer_key: int,  # type: ignore[override]
                clamps: tuple[float, float, float], fp8_pool: nn.Module | None, s_clamps: tuple[float, float, float],
                s_owner: nn.Module | None, *ws: Tensor) -> Tensor:
        from saint_llm_b200.ops.moe_native import shared_group_forward

        wg, wu, wd = ws[:3]
        sws = list(ws[3:])
        call = EPCall(comm, layer_key, h, idx, gate, wg, wu, wd, clamps, fp8_pool)
        main, side = torch.cuda.current_stream(h.device), comm.side
        side.wait_stream(main)
        with torch.cuda.stream(side), _phase("ep.dispatch"):
            call.f1_counts()
            call.f2_dispatch()
        with _phase("moe.shared_fwd"):
            ys, saved = shared_group_forward(h, s_clamps, s_owner, sws)
        main.wait_stream(side)
        with _phase("ep.experts_fwd"):
            call.f3_experts()
        with _phase("ep.combine"):
            out = call.f4_combine()
        out += ys
        ctx.call, ctx.saved_shared, ctx.s_clamps, ctx.n_sws = call, saved, s_clamps, len(sws)
        ctx.save_for_backward(*sws)
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        from saint_llm_b200.ops.moe_native import shared_group_backward

        call: EPCall = ctx.call
        sws = list(ctx.saved_tensors)
        main, side = torch.cuda.current_stream(dout.device), call.comm.side
        dgate = torch.empty_like(call.gf)
        doutb = _bf16c(dout)
        side.wait_stream(main)
        with torch.cuda.stream(side), _phase("ep.combine_bwd"):
            call.b1_push(doutb, dgate)
        with _phase("moe.shared_bwd"):
            dh_s, sgrads = shared_group_backward(ctx.saved_shared, sws, ctx.s_clamps, doutb)
        main.wait_stream(side)
        with _phase("ep.experts_bwd"):
            call.b2_experts()
        with _phase("ep.dispatch_bwd"):
            dh, dgate, dwg, dwu, dwd = call.b3_pull()
        dh += dh_s
        del ctx.call, ctx.saved_shared
        return (dh, None, dgate, None, None, None, None, None, None, dwg, dwu, dwd, *sgrads)


def p2p_routed_experts(h: Tensor, idx: Tensor, gate: Tensor, experts: nn.Module, comm: P2PExpertComm,
                       layer_key: int) -> Tensor:
    """h (T, D) this rank's tokens; idx / gate (T, k) with global expert ids.  Returns
    sum_j gate[t,j] * expert_{idx[t,j]}(h[t]) with the experts sharded over the group."""
    from saint_llm_b200.ops.moe_native import fp8_pool_ok

    return _P2PExpertsFn.apply(h, idx, gate, experts.gate_weight, experts.up_weight, experts.down_weight, comm,
                               layer_key, (float(experts.clamp_gate_max), float(experts.clamp_linear[0]),
                                           float(experts.clamp_linear[1])), experts if fp8_pool_ok(experts) else None)


def moe_forward_p2p(layer: nn.Module, x: Tensor, token_ids: Tensor | None, is_visual: Tensor | None) -> Tensor:
    from saint_llm_b200.ops.moe_native import fp8_pool_ok, shared_experts, shared_group_args

    b, t, d = x.shape
    h = layer.norm(x)
    idx, gate, aux = layer.route(h, token_ids, is_visual)
    layer._last_aux_loss = aux
    k = layer.cfg.experts_per_token
    h2 = h.reshape(b * t, d)
    comm: P2PExpertComm = layer.ep_comm
    shared = shared_group_args(h2, layer.shared_experts)
    if comm.side is not None and shared is not None and getattr(comm, "overlap", True):
        ex = layer.grouped_experts
        s_clamps, s_owner, sws = shared
        out = _P2PMoEFn.apply(h2, idx.reshape(b * t, k), gate.reshape(b * t, k), comm, layer.layer_idx,
                              (float(ex.clamp_gate_max), float(ex.clamp_linear[0]), float(ex.clamp_linear[1])),
                              ex if fp8_pool_ok(ex) else None, s_clamps, s_owner, ex.gate_weight, ex.up_weight,
                              ex.down_weight, *sws)
        return out.view(b, t, d)
    out = p2p_routed_experts(h2, idx.reshape(b * t, k), gate.reshape(b * t, k), layer.grouped_experts,
                             layer.ep_comm, layer.layer_idx)
    sh = shared_experts(h2, layer.shared_experts)
    if sh is not None:
        out = out + sh
    return out.view(b, t, d)


def attach_p2p_comm(model: nn.Module, group: dist.ProcessGroup | None, device: torch.device, *,
                    capacity_factor: float | None = None, timeout_s: float = 30.0) -> P2PExpertComm | None:
    """Give every expert-parallel MoE layer of ``model`` one shared peer-memory communicator."""
    from saint_llm_b200.models.moe import DeepSeekMoE

    layers = [m for m in model.modules() if isinstance(m, DeepSeekMoE) and getattr(m, "ep_size", 1) > 1]
    if not layers:
        return None
    cfg = layers[0].cfg
    comm = P2PExpertComm(SymmetricHeap(group, device), n_experts=cfg.routed_experts,
                         hidden=layers[0].grouped_experts.down_weight.shape[1], top_k=cfg.experts_per_token,
                         capacity_factor=capacity_factor, timeout_s=timeout_s)
    for m in layers:
        m.ep_comm = comm
    model.ep_comm = comm  # callers release it with model.ep_comm.close() (collective)
    return comm


__all__ = ["EPCall", "EmulatedHeap", "FORWARD_STAGES", "P2PExpertComm", "SymmetricBuffer", "SymmetricHeap", "attach_p2p_comm", "moe_forward_p2p",
           "p2p_routed_experts"]

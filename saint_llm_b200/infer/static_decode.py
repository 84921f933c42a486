"""Static-shape greedy decoding with a CUDA-graph-captured step.

The cached decode path (``infer.generate``) re-slices growing caches and takes Python
integer positions, so each step has new shapes and hundreds of host launches.  Here
every buffer has a fixed shape and the position lives on the device, so one decode
step -- 28 layers of attention over the heterogeneous cache, mHC, MoE, final norm, LM
head and argmax -- is a fixed sequence of kernels that is captured once into a CUDA
graph and replayed per token:

* window K/V: a ring of ``sliding_window_size`` slots per layer, written at
  ``pos % W``; a slot is visible iff its position ``pos - age`` is >= 0 (all live slots
  are inside the window by construction);
* compressed streams (HCA / CSA, and the CSA indexer's keys): per-token compressor
  projections of the unfinished block in a ring of ``m`` slots; every step pools them and
  writes the block entry -- the value only becomes visible to later queries once the
  block is complete (block s is visible from position t iff ``s*m + m - 1 < t``), so the
  entry of an unfinished block is simply rewritten until it completes;
* HCA attends to all ``max_len / m'`` entries under that mask; CSA's indexer scores all
  ``max_len / m`` blocks under it and keeps ``min(top_k, blocks)`` picks (picks of
  invisible blocks become -1), then runs the module's own sparse branch.

``StaticDecoder.load(bundle)`` imports the state of a ``KVCacheBundle`` after a prefill
through the cached path.  Outputs equal the cached path's (tested on CPU).
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.kv_cache import CompressedKVLayer, KVCacheBundle
from saint_llm_b200.models.attention import CSA, HCA, SWAttention
from saint_llm_b200.models.attention.common import rope_tables, scaled_dot_product
from saint_llm_b200.models.mhc import MHC
from saint_llm_b200.ops import backend
from saint_llm_b200.ops import decode as decode_ops


class _Ring:
    """Per-token compressor projections of the unfinished block plus the pooled entries."""

    def __init__(self, comp: nn.Module, b: int, n_blocks: int, dev: torch.device, dt: torch.dtype) -> None:
        self.comp = comp
        self.m, c = comp.m, comp.c
        self.cb = torch.zeros(b, self.m, c, device=dev, dtype=dt)
        self.zb = torch.zeros(b, self.m, c, device=dev, dtype=dt)
        self.entries = torch.zeros(b, n_blocks, c, device=dev, dtype=dt)

    def push(self, h: Tensor, pos: Tensor) -> None:
        slot = (pos % self.m).view(1)
        self.cb.index_copy_(1, slot, self.comp.w_b_kv(h).to(self.cb.dtype))
        self.zb.index_copy_(1, slot, self.comp.w_b_z(h).to(self.zb.dtype))
        # slots past the current one still hold the previous block; the pooled value of an
        # unfinished block is never visible, and it is final once slot m-1 is written
        pooled = self.comp.pool(self.cb, self.zb).to(self.entries.dtype)  # (B, 1, c)
        self.entries.index_copy_(1, (pos // self.m).view(1), pooled)

    def load(self, entries: Tensor, raw_tail: Tensor) -> None:
        n = entries.shape[1]
        self.entries[:, :n] = entries.to(self.entries.dtype)
        if raw_tail.shape[1]:
            t = raw_tail.shape[1]
            self.cb[:, :t] = self.comp.w_b_kv(raw_tail).to(self.cb.dtype)
            self.zb[:, :t] = self.comp.w_b_z(raw_tail).to(self.zb.dtype)


class _LayerState:
    def __init__(self, attn: nn.Module, b: int, max_len: int, dev: torch.device, dt: torch.dtype) -> None:
        cfg = attn.attn_cfg
        self.attn = attn
        self.W = cfg.sliding_window_size
        hd = cfg.head_dim
        self.k = torch.zeros(b, self.W, hd, device=dev, dtype=dt)
        self.v = torch.zeros(b, self.W, hd, device=dev, dtype=dt)
        self.kv: _Ring | None = None
        self.idx: _Ring | None = None
        if isinstance(attn, (HCA, CSA)):
            m = attn.kv_compressor.m
            self.kv = _Ring(attn.kv_compressor, b, (max_len + m - 1) // m, dev, dt)
        if isinstance(attn, CSA):
            mi = attn.indexer.compressor.m
            self.idx = _Ring(attn.indexer.compressor, b, (max_len + mi - 1) // mi, dev, dt)
        # fp32 copies of the sink logits and the entry-norm weight for the native kernel
        # (inference weights are fixed while a decoder lives)
        sink = getattr(attn, "sink_logit", None)
        self.sink = None if sink is None else sink.detach().float().contiguous()
        norm = getattr(attn, "k_norm", None)
        self.norm_w = None if norm is None else norm.weight.detach().float().contiguous()


def _attend_layer(st: _LayerState, h: Tensor, pos: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Decode attention of one layer for h (B, 1, D) at device position ``pos``: one native
    kernel on CUDA (``ops.decode``), the eager composition otherwise."""
    a = st.attn
    cfg = a.attn_cfg
    if not (backend.native_for(h) and decode_ops.supported(cfg.head_dim, cfg.query_heads)):
        return _attend_layer_eager(st, h, pos, cos, sin)
    q = a._queries(h, cos, sin)
    k, v = a._sw_kv(h, cos, sin)
    slot = (pos % st.W).view(1)
    st.k.index_copy_(1, slot, k.to(st.k.dtype))
    st.v.index_copy_(1, slot, v.to(st.v.dtype))
    kw = {"sink": st.sink, "softcap": cfg.logit_softcap}
    if st.kv is not None:
        st.kv.push(h, pos)
        kw.update(entries=st.kv.entries, norm_weight=st.norm_w, norm_eps=a.k_norm.eps, m=st.kv.m)
        if isinstance(a, HCA):
            kw.update(mode=1, comp_sink=st.sink)
        else:
            assert st.idx is not None
            st.idx.push(h, pos)
            kw.update(mode=2, top=_indexer_topk(a, st, h, pos))
    return a.output(decode_ops.decode_attention(q, st.k, st.v, pos, **kw))


def _indexer_topk(a: nn.Module, st: _LayerState, h: Tensor, pos: Tensor) -> Tensor:
    """CSA lightning-indexer picks of the visible blocks (B, 1, k); -1 = none."""
    assert st.idx is not None
    idx = a.indexer
    n = st.idx.entries.shape[1]
    m = st.kv.m if st.kv is not None else st.idx.m
    visible = (torch.arange(n, device=h.device) * m + (m - 1) < pos).view(1, n)
    bq = h.shape[0]
    qi = idx.w_iuq(idx.w_dq(h)).view(bq, 1, idx.n_heads, idx.c_indexer)
    w = idx.w_w(h)
    head = torch.einsum("bthc,bnc->bthn", qi, st.idx.entries.to(qi.dtype)).clamp(min=0.0)
    s = (w.unsqueeze(-1) * head).sum(dim=-2)
    s = s.masked_fill(~visible.view(1, 1, n), float("-inf"))
    vals, top = s.topk(min(idx.top_k, n), dim=-1)
    return torch.where(torch.isfinite(vals), top, torch.full_like(top, -1))


def _attend_layer_eager(st: _LayerState, h: Tensor, pos: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """The same step as ``_attend_layer`` in plain PyTorch (the oracle)."""
    a = st.attn
    cfg = a.attn_cfg
    q = a._queries(h, cos, sin)
    k, v = a._sw_kv(h, cos, sin)
    slot = (pos % st.W).view(1)
    st.k.index_copy_(1, slot, k.to(st.k.dtype))
    st.v.index_copy_(1, slot, v.to(st.v.dtype))
    age = (slot - torch.arange(st.W, device=h.device)) % st.W
    live = (age <= pos).view(1, st.W)
    out = scaled_dot_product(q, st.k.unsqueeze(1), st.v.unsqueeze(1), mask=live, sink_logit=a.sink_logit,
                             logit_softcap=cfg.logit_softcap)
    if st.kv is not None:
        st.kv.push(h, pos)
        m = st.kv.m
        n = st.kv.entries.shape[1]
        visible = (torch.arange(n, device=h.device) * m + (m - 1) < pos).view(1, n)
        if isinstance(a, HCA):
            ck = a.k_norm(st.kv.entries).unsqueeze(1)
            comp = scaled_dot_product(q, ck, ck, mask=visible, sink_logit=a.sink_logit)
            if a.sink_logit is None:
                comp = torch.where(visible.any(-1).view(1, 1, 1, 1), comp, torch.zeros_like(comp))
            out = out + comp
        else:
            assert st.idx is not None
            st.idx.push(h, pos)
            out = out + a.sparse_branch(q, st.kv.entries, _indexer_topk(a, st, h, pos))
    return a.output(out)


class StaticDecoder:
    """Greedy decoding with fixed-shape state; ``graph=True`` captures the step (CUDA)."""

    def __init__(self, model: nn.Module, batch: int, max_len: int) -> None:
        self.model = model
        cfg = model.cfg  # type: ignore[attr-defined]
        for blk in model.blocks:  # type: ignore[attr-defined]
            if not isinstance(blk.attention, (SWAttention, HCA, CSA)):
                raise ValueError("static decoding supports SWA / HCA / CSA layers")
        if cfg.n_sink_tokens:
            raise ValueError("static decoding does not support prepended sink tokens")
        p = next(model.parameters())
        self.dev, self.dt = p.device, p.dtype
        self.B, self.max_len = batch, max_len
        self.layers = [_LayerState(blk.attention, batch, max_len, self.dev, self.dt)
                       for blk in model.blocks]  # type: ignore[attr-defined]
        rd = cfg.attention.rope_dim
        self.cos, self.sin = rope_tables(max_len, rd, cfg.attention.rope_theta, self.dev)
        self.pos = torch.zeros((), dtype=torch.long, device=self.dev)
        self.tok = torch.zeros(batch, 1, dtype=torch.long, device=self.dev)
        self.next_tok = torch.zeros(batch, 1, dtype=torch.long, device=self.dev)
        self.logits = torch.zeros(batch, cfg.vocab_size, dtype=torch.float32, device=self.dev)
        self.graph: torch.cuda.CUDAGraph | None = None

    @torch.no_grad()
    def load(self, bundle: KVCacheBundle, last_logits: Tensor) -> None:
        """Import the cache after a prefill of ``bundle.length`` tokens; the first token to
        feed is the argmax of ``last_logits`` (B, V)."""
        length = bundle.length
        if length + 1 > self.max_len:
            raise ValueError("prefill longer than max_len")
        for i, st in enumerate(self.layers):
            c = bundle.for_layer(i)
            lo = max(0, length - st.W)
            slots = torch.arange(lo, length, device=self.dev) % st.W
            st.k[:, slots] = c.k[:, lo:length].to(self.dt)
            st.v[:, slots] = c.v[:, lo:length].to(self.dt)
            if st.kv is not None:
                assert isinstance(c, CompressedKVLayer)
                tail = c.h_buffer
                st.kv.load(c.streams[0][:, :c.n_blocks], tail)
                if st.idx is not None:
                    st.idx.load(c.streams[1][:, :c.n_blocks], tail)
        self.pos.fill_(length)
        self.tok.copy_(last_logits.argmax(-1, keepdim=True))

    def _step(self) -> None:
        m = self.model
        cfg = m.cfg  # type: ignore[attr-defined]
        ids = self.tok
        h = m._embed_inputs(ids, None, None)  # type: ignore[attr-defined]
        x = MHC.expand(h, cfg.mhc.expansion_factor)
        vis = ids == cfg.tokenizer_slots.image_pad
        cos = self.cos.index_select(0, self.pos.view(1))
        sin = self.sin.index_select(0, self.pos.view(1))
        for blk, st in zip(m.blocks, self.layers, strict=True):  # type: ignore[attr-defined]
            inner, _, b_l, c_l = blk.attn_mhc.split(x)
            x = blk.attn_mhc.combine(x, _attend_layer(st, inner, self.pos, cos, sin), b_l, c_l)
            inner, _, b_l, c_l = blk.moe_mhc.split(x)
            x = blk.moe_mhc.combine(x, blk.moe(inner, token_ids=ids, is_visual=vis), b_l, c_l)
            if blk.side_channel.active:
                collapsed = x.mean(-2)
                x = x + ((blk.side_channel(collapsed) - collapsed) / x.shape[-2]).unsqueeze(-2)
        hN = m.final_norm(MHC.collapse(x))  # type: ignore[attr-defined]
        logits = m.logits(hN[:, -1:]).squeeze(1)  # type: ignore[attr-defined]
        self.logits.copy_(logits)
        self.next_tok.copy_(logits.argmax(-1, keepdim=True))
        self.pos.add_(1)

    @torch.no_grad()
    def capture(self, warmup: int = 2) -> None:
        """Capture one step into a CUDA graph (warm-up steps run eagerly on a side stream
        and are undone: positions and caches are restored)."""
        saved = self._snapshot()
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self._restore(saved)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self._restore(saved)

    def _snapshot(self) -> list[Tensor]:
        return [t.clone() for t in self._state()]

    def _restore(self, saved: list[Tensor]) -> None:
        for t, v in zip(self._state(), saved, strict=True):
            t.copy_(v)

    def _state(self) -> list[Tensor]:
        out = [self.pos, self.tok, self.next_tok, self.logits]
        for st in self.layers:
            out += [st.k, st.v]
            for r in (st.kv, st.idx):
                if r is not None:
                    out += [r.cb, r.zb, r.entries]
        return out

    @torch.no_grad()
    def generate(self, steps: int, out: Tensor | None = None) -> Tensor:
        """Greedy ids (B, steps): the fed token of each step (the first is the prefill's
        argmax)."""
        if out is None:
            out = torch.empty(self.B, steps, dtype=torch.long, device=self.dev)
        for i in range(steps):
            out[:, i:i + 1] = self.tok
            if self.graph is not None:
                self.graph.replay()
            else:
                self._step()
            self.tok.copy_(self.next_tok)
        return out


def static_greedy_decode(model: nn.Module, prompt_ids: Tensor, *, max_new_tokens: int, prefill_chunk: int = 256,
                         graph: bool | None = None) -> Tensor:
    """(B, T + max_new_tokens) greedy ids: chunked cached prefill, then static steps."""
    from saint_llm_b200.infer.generate import last_logits

    b, t = prompt_ids.shape
    bundle = KVCacheBundle.for_model(model, max_seq_len=t + max_new_tokens, batch_size=b,
                                     device=prompt_ids.device, keep_history=False)
    logits = None
    with torch.no_grad():
        for c in range(0, t, prefill_chunk):
            logits = last_logits(model, prompt_ids[:, c:c + prefill_chunk], bundle=bundle)
    dec = StaticDecoder(model, b, t + max_new_tokens)
    dec.load(bundle, logits)
    del bundle
    if graph is None:
        graph = prompt_ids.is_cuda
    if graph:
        dec.capture()
    new = dec.generate(max_new_tokens)
    return torch.cat([prompt_ids, new], dim=1)


__all__ = ["StaticDecoder", "static_greedy_decode"]

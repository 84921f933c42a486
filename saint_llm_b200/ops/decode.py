"""Native single-token decode attention over the heterogeneous cache (one kernel per layer).

``decode_attention`` computes, for every sequence and query head, the sliding-window
branch (ring of W slots, live iff the slot's age is <= pos, softcap, optional sink) plus
the compressed branch (HCA: every visible entry, optional sink; CSA: the listed top-k
entries), with K = V = RMSNorm(entry) applied on the fly.  The eager composition it
replaces is ``infer.static_decode._attend_layer_eager``.

``decode_attention_paged`` is the serving variant: sequences of different lengths decode in
one launch, and the K / V stream and the compressed entries are read through per-sequence
block tables from the shared page pools of ``infer.paged_kv`` (no gather into contiguous
buffers first).
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from saint_llm_b200.ops import backend


def supported(head_dim: int, heads: int) -> bool:
    return head_dim == 128 and heads % 4 == 0


def decode_attention(q: Tensor, k_win: Tensor, v_win: Tensor, pos: Tensor, *, sink: Tensor | None,
                     softcap: float | None, mode: int = 0, entries: Tensor | None = None,
                     norm_weight: Tensor | None = None, norm_eps: float = 1e-6, m: int = 0,
                     top: Tensor | None = None, comp_sink: Tensor | None = None) -> Tensor:
    """q (B, H, 1, 128); k_win / v_win (B, W, 128); pos: int64 device scalar.
    mode 0: window only; 1: + HCA entries (B, n, 128) with compression rate ``m``;
    2: + CSA entries gathered by ``top`` (B, k) int64 (-1 = none).  Returns (B, H, 1, 128)."""
    b, h, _, d = q.shape
    out = torch.empty(b, h, 1, d, dtype=torch.bfloat16, device=q.device)
    backend.ext().decode_attention(
        q.reshape(b, h, d).to(torch.bfloat16).contiguous(), k_win, v_win, pos,
        None if sink is None else sink.float().contiguous(), float(softcap or 0.0), mode,
        entries, None if norm_weight is None else norm_weight.float().contiguous(), float(norm_eps), int(m),
        None if top is None else top.reshape(b, -1).contiguous(),
        None if comp_sink is None else comp_sink.float().contiguous(), 1.0 / math.sqrt(d), out)
    return out


def decode_attention_paged(q: Tensor, k_pool: Tensor, v_pool: Tensor, k_table: Tensor, k_len: Tensor, *,
                           window: int = 0, sink: Tensor | None = None, softcap: float | None = None,
                           mode: int = 0, e_pool: Tensor | None = None, e_table: Tensor | None = None,
                           e_len: Tensor | None = None, norm_weight: Tensor | None = None, norm_eps: float = 1e-6,
                           m: int = 0, top: Tensor | None = None, comp_sink: Tensor | None = None,
                           max_rows: int | None = None, splits: int = 1) -> Tensor:
    """q (B, H, 128) or (B, H, 1, 128); k_pool / v_pool (pages, page_rows, 128) bf16 storages;
    k_table (B, P) int32 block tables (-1 padded), k_len (B,) int32 rows per sequence (the
    current token included).  The window branch attends to the last ``window`` rows (0: all).
    mode 1 / 2 add the compressed branch over the entry stream (``e_pool`` / ``e_table`` /
    ``e_len``): HCA with compression rate ``m``, or the CSA entries listed in ``top`` (B, k).
    ``max_rows`` bounds any branch's length (default: the longest ``k_len`` / ``e_len``, read
    on the host).  Returns (B, H, 128) bf16.  A page id outside the pool records the bounds
    error (``gemm.check_errors``) and the row is skipped.  ``splits > 1`` spreads each
    sequence's window rows over that many CTAs (partial max / sum / output per slice) and merges
    them with ``lse_merge``: for long windows at small batch."""
    from saint_llm_b200.ops.gemm import error_word

    b, h = q.shape[0], q.shape[1]
    d = q.shape[-1]
    if splits > 1:
        kmax = int(k_len.max().item()) if k_len.numel() else 1
        wrows = max(1, min(kmax, window) if window > 0 else kmax)
        qb = q.reshape(b, h, d).to(torch.bfloat16).contiguous()
        pm = torch.empty(splits, b * h, dtype=torch.float32, device=q.device)
        pl = torch.empty_like(pm)
        po = torch.empty(splits, b * h, d, dtype=torch.float32, device=q.device)
        backend.ext().decode_window_split(qb, k_pool, v_pool, k_table.int().contiguous(), k_len.int().contiguous(),
                                          int(window), float(softcap or 0.0), 1.0 / math.sqrt(d), int(splits), wrows,
                                          pm, pl, po, error_word(q.device))
        win = lse_merge(pm, pl, po, extra=None if sink is None else sink.float().contiguous())[2].view(b, h, d)
        if mode == 0:
            return win.to(torch.bfloat16)
        comp = decode_attention_paged(q, k_pool, v_pool, k_table, k_len, window=-1, softcap=softcap, mode=mode,
                                      e_pool=e_pool, e_table=e_table, e_len=e_len, norm_weight=norm_weight,
                                      norm_eps=norm_eps, m=m, top=top, comp_sink=comp_sink, max_rows=max_rows)
        return (win + comp.float()).to(torch.bfloat16)
    if max_rows is None:
        rows = [int(k_len.max().item()) if k_len.numel() else 1]
        if window > 0:
            rows = [min(rows[0], window)]
        if mode == 1 and e_len is not None and e_len.numel():
            rows.append(int(e_len.max().item()))
        max_rows = max(1, *rows)
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device=q.device)
    backend.ext().decode_attention_paged(
        q.reshape(b, h, d).to(torch.bfloat16).contiguous(), k_pool, v_pool, k_table.int().contiguous(),
        k_len.int().contiguous(), int(window), None if sink is None else sink.float().contiguous(),
        float(softcap or 0.0), mode, e_pool, None if e_table is None else e_table.int().contiguous(),
        None if e_len is None else e_len.int().contiguous(),
        None if norm_weight is None else norm_weight.float().contiguous(), float(norm_eps), int(m),
        None if top is None else top.reshape(b, -1).long().contiguous(),
        None if comp_sink is None else comp_sink.float().contiguous(), 1.0 / math.sqrt(d), int(max_rows), out,
        error_word(q.device))
    return out


def lse_merge(m: Tensor, l: Tensor, o: Tensor, *, extra: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:  # noqa: E741
    """Associative merge of S attention partials in one kernel: ``m``, ``l`` (S, ...) row max
    and sum of exponentials, ``o`` (S, ..., D) normalised outputs (fp32).  ``extra``: an
    optional logit per row joining only the denominator (a sink; row r uses
    ``extra[r % extra.numel()]``).  Returns the merged (m, l, o); rows with nothing to attend
    give o = 0, l = 0."""
    s_, lead, d = m.shape[0], m.shape[1:], o.shape[-1]
    r = m[0].numel()
    out = torch.empty(r, d, dtype=torch.float32, device=o.device)
    om = torch.empty(r, dtype=torch.float32, device=o.device)
    ol = torch.empty_like(om)
    backend.ext().lse_merge(m.float().reshape(s_, r).contiguous(), l.float().reshape(s_, r).contiguous(),
                            o.float().reshape(s_, r, d).contiguous(), extra, out, om, ol)
    return om.view(lead), ol.view(lead), out.view(*lead, d)


__all__ = ["decode_attention", "decode_attention_paged", "lse_merge", "supported"]

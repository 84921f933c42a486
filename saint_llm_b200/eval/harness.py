"""lm-eval-harness style adapter (reference: ``saint_llm_eval/harness/saint_llm_lm.py:46-173``):
``loglikelihood`` -> (sum log p(continuation | context), continuation is the greedy one),
``loglikelihood_rolling`` -> total log p(text), ``generate_until`` -> greedy text cut at the
first stop string.  Requests only need an ``args`` tuple (duck-typed ``Instance``).

Scoring requests are batched: right-padded rows run one backbone pass and the LM head is
applied only at the scored positions."""

from __future__ import annotations

from typing import Any, Protocol

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from saint_llm_b200.data.tokenizer import Tokenizer
from saint_llm_b200.infer.generate import greedy_decode_cached


class _Request(Protocol):
    args: tuple[Any, ...]


class SaintLLMHarnessLM:
    def __init__(self, *, model: nn.Module, tokenizer: Tokenizer, device: torch.device | str = "cpu",
                 max_length: int = 4096, batch_size: int = 16) -> None:
        self.model, self.tokenizer = model, tokenizer
        self.device = torch.device(device)
        self.max_length, self.batch_size = max_length, batch_size

    @property
    def eot_token_id(self) -> int:
        return self.tokenizer.eos_token_id

    # ---- scoring core: rows of ids, each with the span [lo, len) scored ------------------
    def _score_rows(self, rows: list[list[int]], spans: list[int]) -> list[tuple[float, bool]]:
        out: list[tuple[float, bool]] = []
        order = sorted(range(len(rows)), key=lambda i: len(rows[i]))
        res: dict[int, tuple[float, bool]] = {}
        for b0 in range(0, len(order), self.batch_size):
            idx = order[b0:b0 + self.batch_size]
            width = max(len(rows[i]) for i in idx)
            toks = torch.zeros(len(idx), width, dtype=torch.long)
            for j, i in enumerate(idx):
                toks[j, :len(rows[i])] = torch.tensor(rows[i])
            toks = toks.to(self.device)
            pos_r, pos_t, tgt = [], [], []
            for j, i in enumerate(idx):
                n = len(rows[i])
                for p in range(n - spans[i], n):  # predict token p from position p - 1
                    pos_r.append(j)
                    pos_t.append(p - 1)
                    tgt.append(rows[i][p])
            logits = self._logits_at(toks, torch.tensor(pos_r, device=self.device),
                                     torch.tensor(pos_t, device=self.device))
            lp = F.log_softmax(logits.float(), -1)
            tgt_t = torch.tensor(tgt, device=self.device)
            tok_lp = lp.gather(-1, tgt_t[:, None]).squeeze(-1)
            greedy = lp.argmax(-1) == tgt_t
            k = 0
            for i in idx:
                s = spans[i]
                res[i] = (float(tok_lp[k:k + s].sum()), bool(greedy[k:k + s].all()))
                k += s
        for i in range(len(rows)):
            out.append(res[i])
        return out

    def _logits_at(self, toks: Tensor, rows: Tensor, cols: Tensor) -> Tensor:
        m = self.model
        if hasattr(m, "backbone") and hasattr(m, "logits"):
            h, _ = m.backbone(toks)
            return m.logits(h[rows, cols])
        return m(toks)["logits"][rows, cols]

    def _eval(self, fn):  # noqa: ANN001
        was = self.model.training
        self.model.eval()
        try:
            with torch.no_grad():
                return fn()
        finally:
            self.model.train(was)

    def loglikelihood(self, requests: list[_Request]) -> list[tuple[float, bool]]:
        rows, spans, trivial = [], [], {}
        for qi, req in enumerate(requests):
            ctx, cont = (str(a) for a in req.args)
            full = self.tokenizer.encode(ctx) + (cont_ids := self.tokenizer.encode(cont))
            full = full[-self.max_length:]
            n = min(len(cont_ids), len(full) - 1)
            if not cont_ids or n <= 0:
                trivial[qi] = (0.0, True)
                continue
            rows.append(full)
            spans.append(n)
        scored = iter(self._eval(lambda: self._score_rows(rows, spans)) if rows else [])
        return [trivial[i] if i in trivial else next(scored) for i in range(len(requests))]

    def loglikelihood_rolling(self, requests: list[_Request]) -> list[float]:
        rows, spans, trivial = [], [], {}
        for qi, req in enumerate(requests):
            ids = self.tokenizer.encode(str(req.args[0]))[: self.max_length]
            if len(ids) < 2:
                trivial[qi] = 0.0
                continue
            rows.append(ids)
            spans.append(len(ids) - 1)
        scored = iter(self._eval(lambda: self._score_rows(rows, spans)) if rows else [])
        return [trivial[i] if i in trivial else next(scored)[0] for i in range(len(requests))]

    def generate_until(self, requests: list[_Request]) -> list[str]:
        def run() -> list[str]:
            outs = []
            for req in requests:
                ctx, kw = req.args
                kw = kw if isinstance(kw, dict) else {}
                until = [u for u in (kw.get("until") or []) if u]
                ids = self.tokenizer.encode(str(ctx))[-self.max_length:]
                prompt = torch.tensor([ids], device=self.device)
                gen = greedy_decode_cached(self.model, prompt, max_new_tokens=int(kw.get("max_gen_toks", 256)))
                text = self.tokenizer.decode(gen[0, len(ids):].tolist())
                cut = min((text.find(u) for u in until if u in text), default=-1)
                outs.append(text[:cut] if cut >= 0 else text)
            return outs

        return self._eval(run)


__all__ = ["SaintLLMHarnessLM"]

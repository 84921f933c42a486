"""Speculative decoding with a draft head (EAGLE-3 loop; reference:
``saint_llm_inference/eagle3.py:45-204``).

Per round the draft head proposes ``draft_length`` tokens from the base model's last
hidden state; ONE base forward over the proposals verifies them, the longest agreeing
prefix is accepted, and the base model's own token at the first disagreement (or after
the last proposal) is appended.  With a greedy verifier the output therefore equals
greedy decoding of the base model, whatever the draft proposes.

Differences from the reference loop: the verification forward's hidden states seed the
next round, so there is one base forward per round instead of two; the draft head is
run autoregressively on its own proposals (``draft_head(hidden, token)`` when the head
takes the previous token, as a trained EAGLE head does); with ``use_cache=True`` the base
runs through the KV cache and rejected positions are rolled back with
``KVCacheBundle.truncate``; the result is cut to exactly ``max_new_tokens``.
"""

from __future__ import annotations

import inspect
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.kv_cache import KVCacheBundle


@dataclass(frozen=True)
class EAGLE3Config:
    draft_length: int = 4
    temperature: float = 0.0
    max_new_tokens: int = 64
    use_cache: bool = False


class EAGLE3DraftHead(nn.Module):
    """Minimal draft head: hidden (B, T, D) [+ previous token] -> logits (B, T, V)."""

    def __init__(self, hidden_dim: int, vocab_size: int, *, token_conditioned: bool = False) -> None:
        super().__init__()
        self.proj = nn.Linear(hidden_dim, vocab_size, bias=False)
        self.token_embed = nn.Embedding(vocab_size, hidden_dim) if token_conditioned else None
        if self.token_embed is not None:
            nn.init.zeros_(self.token_embed.weight)

    def forward(self, hidden: Tensor, token: Tensor | None = None) -> Tensor:
        if self.token_embed is not None and token is not None:
            hidden = hidden + self.token_embed(token)
        return self.proj(hidden)


def _base(model: nn.Module, ids: Tensor, bundle: KVCacheBundle | None) -> tuple[Tensor, Tensor]:
    """(hidden (B,T,D), logits (B,T,V)) of the base model."""
    if hasattr(model, "backbone"):
        h, _ = model.backbone(ids, kv_cache_bundle=bundle)
        return h, model.logits(h)
    out = model(ids, kv_cache_bundle=bundle) if bundle is not None else model(ids)
    return out["hidden"], out["logits"]


@torch.no_grad()
def speculative_decode(base_model: nn.Module, draft_head: nn.Module, prompt: Tensor, *,
                       cfg: EAGLE3Config) -> tuple[Tensor, dict[str, float]]:
    if prompt.dim() != 2 or prompt.shape[0] != 1:
        raise ValueError(f"speculative_decode requires batch_size=1; got shape {tuple(prompt.shape)}")
    if cfg.draft_length <= 0:
        raise ValueError("draft_length must be positive")
    base_model.eval()
    draft_head.eval()
    takes_token = len(inspect.signature(draft_head.forward).parameters) >= 2
    k = cfg.draft_length
    t0 = prompt.shape[1]
    cap = t0 + cfg.max_new_tokens + k + 1
    ids = torch.empty((1, cap), dtype=prompt.dtype, device=prompt.device)
    ids[:, :t0] = prompt
    n = t0
    sinks = int(getattr(getattr(base_model, "cfg", None), "n_sink_tokens", 0) or 0)
    bundle = KVCacheBundle.for_model(base_model, max_seq_len=cap + sinks, device=prompt.device,
                                     keep_history=True) if cfg.use_cache else None
    hidden, logits = _base(base_model, ids[:, :n], bundle)
    h_last, next_tok = hidden[:, -1:], int(logits[0, -1].argmax())
    drafted = accepted = forwards = 0
    forwards += 1
    while n - t0 < cfg.max_new_tokens:
        ids[0, n] = next_tok  # the base model's own token is always correct
        n += 1
        # draft k tokens autoregressively on the draft head
        prev = ids[:, n - 1:n]
        props = []
        for _ in range(k):
            dl = draft_head(h_last, prev) if takes_token else draft_head(h_last)
            if cfg.temperature == 0.0:
                tok = dl[0, -1].argmax()
            else:
                tok = torch.multinomial(torch.softmax(dl[0, -1].float() / cfg.temperature, -1), 1)[0]
            props.append(tok)
            prev = tok.view(1, 1)
        prop = torch.stack(props).view(1, k).to(ids.dtype)
        ids[:, n:n + k] = prop
        drafted += k
        # verify: base logits at positions n-1 .. n+k-1 predict tokens n .. n+k
        if bundle is not None:
            hv, lv = _base(base_model, ids[:, n - 1:n + k], bundle)
        else:
            hv, lv = _base(base_model, ids[:, :n + k], None)
            hv, lv = hv[:, n - 1:], lv[:, n - 1:]
        forwards += 1
        pred = lv[0].argmax(-1)                         # (k+1,)
        agree = (pred[:k] == prop[0]).long().cumprod(0)
        a = int(agree.sum())
        accepted += a
        n += a
        next_tok = int(pred[a])
        h_last = hv[:, a:a + 1]
        if bundle is not None:
            bundle.truncate(sinks + n)
    out = ids[:, :t0 + cfg.max_new_tokens].clone()
    new = cfg.max_new_tokens
    return out, {"acceptance_rate": accepted / max(drafted, 1), "base_forwards": float(forwards),
                 "new_tokens": float(new)}


__all__ = ["EAGLE3Config", "EAGLE3DraftHead", "speculative_decode"]

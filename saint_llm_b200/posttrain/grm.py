"""Generative reward model: an LM judge scored on a few "verdict" tokens at the next
position; reward = expected score value under the renormalised verdict distribution
(reference: ``saint_llm_posttraining/grm.py:45-232``)."""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from saint_llm_b200.infer.generate import last_logits

DEFAULT_BINARY_TEMPLATE = ("Prompt:\n{prompt}\n\nResponse:\n{completion}\n\n"
                           "Was the response correct? Answer with one word: ")


@dataclass(frozen=True)
class GRMConfig:
    prompt_template: str
    score_token_ids: tuple[int, ...]
    score_values: tuple[float, ...]
    temperature: float = 1.0

    def __post_init__(self) -> None:
        if len(self.score_token_ids) != len(self.score_values):
            raise ValueError("score_token_ids and score_values must have the same length")
        if not self.score_token_ids:
            raise ValueError("at least one score token is required")
        if self.temperature <= 0.0:
            raise ValueError(f"temperature must be positive; got {self.temperature}")


def judge_completion(judge: nn.Module, tokens: Tensor, cfg: GRMConfig) -> Tensor:
    """(B, T) rendered judge prompts -> (B,) expected score (only the last position's logits are computed)."""
    if tokens.dim() != 2:
        raise ValueError(f"tokens must be (B, T); got shape {tuple(tokens.shape)}")
    last = last_logits(judge, tokens).float()
    ids = torch.tensor(cfg.score_token_ids, device=last.device)
    probs = torch.softmax(last.index_select(-1, ids) / cfg.temperature, -1)
    return probs @ torch.tensor(cfg.score_values, device=last.device, dtype=probs.dtype)


class GRMRewardFn:
    """(prompt, completion) -> float via a judge LM."""

    def __init__(self, judge: nn.Module, encode: Callable[[str], Sequence[int]], cfg: GRMConfig, *,
                 device: torch.device | None = None) -> None:
        self._judge, self._encode, self._cfg = judge, encode, cfg
        self._device = device or next(judge.parameters(), torch.empty(0)).device

    @torch.no_grad()
    def __call__(self, prompt: str, completion: str) -> float:
        ids = list(self._encode(self._cfg.prompt_template.format(prompt=prompt, completion=completion)))
        if not ids:
            raise ValueError("encoded judge prompt is empty")
        was = self._judge.training
        self._judge.eval()
        try:
            return float(judge_completion(self._judge, torch.tensor([ids], device=self._device), self._cfg)[0])
        finally:
            self._judge.train(was)


def binary_grm_config(*, good_token_id: int, bad_token_id: int, prompt_template: str = DEFAULT_BINARY_TEMPLATE,
                      temperature: float = 1.0) -> GRMConfig:
    return GRMConfig(prompt_template, (good_token_id, bad_token_id), (1.0, 0.0), temperature)


def likert_grm_config(*, score_token_ids: Sequence[int], prompt_template: str, temperature: float = 1.0) -> GRMConfig:
    k = len(score_token_ids)
    if k < 2:
        raise ValueError(f"likert needs at least 2 score tokens; got {k}")
    return GRMConfig(prompt_template, tuple(score_token_ids), tuple(i / (k - 1) for i in range(k)), temperature)


__all__ = ["DEFAULT_BINARY_TEMPLATE", "GRMConfig", "GRMRewardFn", "binary_grm_config", "judge_completion",
           "likert_grm_config"]

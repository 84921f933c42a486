"""Reward functions for captioning RL (reference: ``saint_llm_posttraining/caption_rewards.py``):
unigram-overlap precision / recall / F1 against a reference, a length window with linear
decay, constant, weighted composites and per-prompt reference lookup."""

from __future__ import annotations

from collections.abc import Callable, Sequence

RewardCallable = Callable[[str, str], float]


def _unigrams(text: str) -> set[str]:
    return set(text.lower().split())


def unigram_overlap_reward(prompt: str, completion: str, *, target: str, mode: str = "f1") -> float:
    del prompt
    if mode not in ("f1", "precision", "recall"):
        raise ValueError(f"unknown mode {mode!r}; use 'f1' / 'precision' / 'recall'")
    pred, ref = _unigrams(completion), _unigrams(target)
    common = len(pred & ref)
    if not pred or not ref or not common:
        return 0.0
    p, r = common / len(pred), common / len(ref)
    return {"precision": p, "recall": r, "f1": 2 * p * r / (p + r)}[mode]


def length_target_reward(prompt: str, completion: str, *, target_min: int, target_max: int,
                         decay_tokens: int = 10) -> float:
    del prompt
    if target_min < 0 or target_max < target_min:
        raise ValueError(f"need 0 <= target_min <= target_max; got ({target_min}, {target_max})")
    if decay_tokens < 0:
        raise ValueError(f"decay_tokens must be >= 0; got {decay_tokens}")
    n = len(completion.lower().split())
    if target_min <= n <= target_max:
        return 1.0
    if decay_tokens == 0:
        return 0.0
    dist = target_min - n if n < target_min else n - target_max
    return max(0.0, 1.0 - dist / decay_tokens)


def constant_reward(_prompt: str, _completion: str, *, value: float = 0.0) -> float:
    return float(value)


def composite_caption_reward(components: Sequence[tuple[float, RewardCallable]]) -> RewardCallable:
    parts = [(float(w), f) for w, f in components]
    return lambda prompt, completion: sum(w * f(prompt, completion) for w, f in parts)


class PerExampleCaptionRewardFn:
    def __init__(self, *, prompt_to_targets: dict[str, Sequence[str]], scorer: Callable[[str, str], float],
                 multi_target_reduce: str = "max", missing_prompt_value: float = 0.0) -> None:
        if multi_target_reduce not in ("max", "mean"):
            raise ValueError(f"multi_target_reduce must be 'max' or 'mean'; got {multi_target_reduce!r}")
        self._targets, self._scorer = prompt_to_targets, scorer
        self._reduce, self._missing = multi_target_reduce, float(missing_prompt_value)

    def __call__(self, prompt: str, completion: str) -> float:
        targets = self._targets.get(prompt)
        if not targets:
            return self._missing
        scores = [self._scorer(completion, t) for t in targets]
        return max(scores) if self._reduce == "max" else sum(scores) / len(scores)


__all__ = ["PerExampleCaptionRewardFn", "RewardCallable", "composite_caption_reward", "constant_reward",
           "length_target_reward", "unigram_overlap_reward"]

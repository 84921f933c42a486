"""Trust layer for open / decentralized training (reference: ``saint_llm_distributed/
verification.py``, ``reputation.py``, ``decentralized_round.py``):

* ``GradientVerifier`` re-runs forward/backward on the sample a peer claims to have used and
  compares per-parameter gradients (cosine, norm ratio); accept iff every cosine > 0 and the
  mean cosine >= threshold.  The verifier's own gradient state is saved and restored.
* ``PeerReputationTracker``: EWMA score per peer (clamped to [floor, ceiling]) and a
  reputation-weighted mean of peer gradients (peers under ``min_score`` excluded, uniform
  fallback when no weight is left).
* ``DecentralizedTrainingRound``: verify -> update reputation -> weighted reduce of accepted.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass

import torch
from torch import Tensor, nn

LossFn = Callable[[nn.Module, Tensor, Tensor], Tensor]


@dataclass(frozen=True)
class GradientCheck:
    name: str
    cosine: float
    norm_ratio: float

    @property
    def passes(self) -> bool:
        return math.isfinite(self.cosine) and self.cosine > 0.0


@dataclass(frozen=True)
class VerificationResult:
    accepted: bool
    mean_cosine: float
    min_cosine: float
    checks: tuple[GradientCheck, ...]

    @property
    def reason(self) -> str:
        if self.accepted:
            return "accepted"
        if self.min_cosine <= 0.0:
            return f"rejected: min_cosine={self.min_cosine:.3f} <= 0"
        return f"rejected: mean_cosine={self.mean_cosine:.3f} below threshold"


def _local_grads(model: nn.Module, loss_fn: LossFn, inputs: Tensor, labels: Tensor) -> dict[str, Tensor]:
    saved = {p: p.grad for p in model.parameters()}
    for p in model.parameters():
        p.grad = None
    was = model.training
    try:
        model.eval()
        loss = loss_fn(model, inputs, labels)
        if not isinstance(loss, Tensor):
            raise TypeError(f"loss_fn must return a Tensor; got {type(loss).__name__}")
        loss.backward()
        return {n: (p.grad.detach().clone() if p.grad is not None else torch.zeros_like(p))
                for n, p in model.named_parameters()}
    finally:
        model.train(was)
        for p, g in saved.items():
            p.grad = g


def _cos_and_ratio(a: Tensor, b: Tensor) -> tuple[float, float]:
    a, b = a.detach().reshape(-1).float(), b.detach().reshape(-1).float().to(a.device)
    na, nb = a.norm(), b.norm()
    if float(na) == 0.0 or float(nb) == 0.0:
        return 0.0, 0.0
    return float(a @ b / (na * nb)), float(na / nb)


class GradientVerifier:
    def __init__(self, model: nn.Module, loss_fn: LossFn, *, cosine_threshold: float = 0.95,
                 param_filter: Callable[[str], bool] | None = None) -> None:
        if not 0.0 <= cosine_threshold <= 1.0:
            raise ValueError(f"cosine_threshold must be in [0, 1]; got {cosine_threshold}")
        self._model, self._loss_fn, self._threshold, self._filter = model, loss_fn, cosine_threshold, param_filter

    def verify(self, peer_gradients: Iterable[Tensor], peer_param_names: Sequence[str], *, inputs: Tensor,
               labels: Tensor) -> VerificationResult:
        claims = list(peer_gradients)
        if len(claims) != len(peer_param_names):
            raise ValueError(f"{len(claims)} gradients for {len(peer_param_names)} names")
        local = _local_grads(self._model, self._loss_fn, inputs, labels)
        checks = []
        for name, claim in zip(peer_param_names, claims, strict=True):
            if name not in local or (self._filter is not None and not self._filter(name)):
                continue
            if claim.shape != local[name].shape:
                raise ValueError(f"{name}: claimed shape {tuple(claim.shape)} != {tuple(local[name].shape)}")
            checks.append(GradientCheck(name, *_cos_and_ratio(claim, local[name])))
        if not checks:
            return VerificationResult(False, 0.0, 0.0, ())
        cos = [c.cosine for c in checks]
        mean_c, min_c = sum(cos) / len(cos), min(cos)
        ok = min_c > 0.0 and mean_c >= self._threshold and all(math.isfinite(c) for c in cos)
        return VerificationResult(ok, mean_c, min_c, tuple(checks))


def random_peer_gradient(model: nn.Module, *, scale: float = 1.0, seed: int | None = None
                         ) -> tuple[list[Tensor], list[str]]:
    g = torch.Generator()
    if seed is not None:
        g.manual_seed(seed)
    named = list(model.named_parameters())
    return [torch.randn(p.shape, generator=g) * scale for _, p in named], [n for n, _ in named]


@dataclass(frozen=True)
class PeerReputationConfig:
    initial_score: float = 0.5
    decay: float = 0.95
    floor: float = 0.0
    ceiling: float = 1.0

    def __post_init__(self) -> None:
        if not 0.0 <= self.initial_score <= 1.0:
            raise ValueError("initial_score must be in [0, 1]")
        if not 0.0 <= self.decay < 1.0:
            raise ValueError("decay must be in [0, 1)")
        if not 0.0 <= self.floor <= self.ceiling <= 1.0:
            raise ValueError("need 0 <= floor <= ceiling <= 1")


class PeerReputationTracker:
    def __init__(self, cfg: PeerReputationConfig | None = None) -> None:
        self._cfg = cfg or PeerReputationConfig()
        self._scores: dict[str, float] = {}

    @property
    def cfg(self) -> PeerReputationConfig:
        return self._cfg

    def score(self, peer_id: str) -> float:
        return self._scores.get(peer_id, self._cfg.initial_score)

    def update(self, peer_id: str, *, accepted: bool) -> float:
        c = self._cfg
        new = c.decay * self.score(peer_id) + (1 - c.decay) * (1.0 if accepted else 0.0)
        self._scores[peer_id] = min(c.ceiling, max(c.floor, new))
        return self._scores[peer_id]

    def update_batch(self, peer_ids: Sequence[str], accepted: Sequence[bool]) -> list[float]:
        if len(peer_ids) != len(accepted):
            raise ValueError("peer_ids and accepted must have equal length")
        return [self.update(p, accepted=a) for p, a in zip(peer_ids, accepted, strict=True)]

    def remove(self, peer_id: str) -> bool:
        return self._scores.pop(peer_id, None) is not None

    def all_scores(self) -> dict[str, float]:
        return dict(self._scores)


def reputation_weighted_reduce(peer_gradients: Sequence[Sequence[Tensor]], peer_ids: Sequence[str],
                               tracker: PeerReputationTracker, *, min_score: float = 0.0, eps: float = 1e-8
                               ) -> list[Tensor]:
    if not peer_gradients:
        return []
    if len(peer_gradients) != len(peer_ids):
        raise ValueError("peer_gradients and peer_ids must have equal length")
    n_par = len(peer_gradients[0])
    if any(len(g) != n_par for g in peer_gradients):
        raise ValueError("every peer must submit the same number of parameter gradients")
    w = torch.tensor([s if (s := tracker.score(p)) >= min_score else 0.0 for p in peer_ids], dtype=torch.float64)
    if float(w.sum()) < eps:
        w = torch.ones_like(w)
    w = w / w.sum()
    return [sum(float(w[i]) * peer_gradients[i][j] for i in range(len(peer_ids)) if w[i] > 0) for j in range(n_par)]


@dataclass(frozen=True)
class PeerSubmission:
    peer_id: str
    gradient_claim: list[Tensor]
    parameter_names: list[str]
    sample: Tensor
    label: Tensor


@dataclass(frozen=True)
class PeerOutcome:
    peer_id: str
    accepted: bool
    new_reputation: float
    verification: VerificationResult


@dataclass(frozen=True)
class RoundResult:
    aggregated: list[Tensor]
    parameter_names: list[str]
    outcomes: list[PeerOutcome]
    n_accepted: int


class DecentralizedTrainingRound:
    def __init__(self, *, verifier: GradientVerifier, tracker: PeerReputationTracker, min_score: float = 0.1) -> None:
        self._verifier, self._tracker, self._min_score = verifier, tracker, min_score

    def process(self, submissions: list[PeerSubmission]) -> RoundResult:
        outcomes, grads, ids = [], [], []
        names: list[str] | None = None
        for s in submissions:
            res = self._verifier.verify(s.gradient_claim, s.parameter_names, inputs=s.sample, labels=s.label)
            outcomes.append(PeerOutcome(s.peer_id, res.accepted, self._tracker.update(s.peer_id, accepted=res.accepted),
                                        res))
            if res.accepted:
                if names is None:
                    names = list(s.parameter_names)
                elif list(s.parameter_names) != names:
                    raise ValueError(f"peer {s.peer_id!r} parameter names differ from earlier accepted peers")
                grads.append(list(s.gradient_claim))
                ids.append(s.peer_id)
        if not grads:
            return RoundResult([], [], outcomes, 0)
        agg = reputation_weighted_reduce(grads, ids, self._tracker, min_score=self._min_score)
        return RoundResult(agg, names or [], outcomes, len(grads))


__all__ = ["DecentralizedTrainingRound", "GradientCheck", "GradientVerifier", "PeerOutcome", "PeerReputationConfig",
           "PeerReputationTracker", "PeerSubmission", "RoundResult", "VerificationResult", "random_peer_gradient",
           "reputation_weighted_reduce"]

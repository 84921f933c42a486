"""Bittensor-style miner / validator protocol over JSON-RPC (reference:
``saint_llm_distributed/bittensor.py:55-303``): miners serve ``ping``, ``miner/info`` and
``miner/serve``; validators query every miner, score responses and normalise scores into
weights; cohort-consensus scoring and multi-validator aggregation helpers."""

from __future__ import annotations

import statistics
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any, Protocol

from saint_llm_b200.agents.jsonrpc import JsonRpcChannel, JsonRpcServer, RpcError, INVALID_PARAMS


class MinerHandler(Protocol):
    def serve(self, query: str) -> str: ...


class ValidatorScorer(Protocol):
    def score(self, query: str, response: str) -> float: ...


@dataclass(frozen=True)
class MinerInfo:
    uid: str
    name: str = ""
    description: str = ""
    metadata: Mapping[str, Any] | None = None


@dataclass(frozen=True)
class MinerResponse:
    uid: str
    query: str
    response: str
    error: str | None = None


@dataclass(frozen=True)
class WeightedScore:
    uid: str
    raw_score: float
    weight: float
    response: str


class BittensorMinerServer(JsonRpcServer):
    def __init__(self, handler: MinerHandler, info: MinerInfo) -> None:
        self._handler, self._info = handler, info
        self.methods = {"ping": lambda p: {}, "miner/info": self._meta, "miner/serve": self._serve}

    def _meta(self, params: Mapping[str, Any]) -> dict[str, Any]:
        i = self._info
        return {"uid": i.uid, "name": i.name, "description": i.description, "metadata": dict(i.metadata or {})}

    def _serve(self, params: Mapping[str, Any]) -> dict[str, Any]:
        q = params.get("query")
        if not isinstance(q, str):
            raise RpcError(INVALID_PARAMS, "miner/serve requires a string 'query'")
        return {"uid": self._info.uid, "response": str(self._handler.serve(q))}


class BittensorValidatorClient:
    def __init__(self, *, scorer: ValidatorScorer, channels: Mapping[str, JsonRpcChannel]) -> None:
        self._scorer, self._channels, self._next = scorer, dict(channels), 1

    def query_all(self, query: str) -> list[MinerResponse]:
        out = []
        for uid, ch in self._channels.items():
            mid, self._next = self._next, self._next + 1
            ch.send({"jsonrpc": "2.0", "id": mid, "method": "miner/serve", "params": {"query": query}})
            reply = None
            while (msg := ch.receive()) is not None:
                if msg.get("id") == mid:
                    reply = msg
                    break
            if reply is None:
                out.append(MinerResponse(uid, query, "", "channel closed before reply"))
            elif "error" in reply:
                e = reply["error"]
                out.append(MinerResponse(uid, query, "", f"{e.get('code')}: {e.get('message')}"))
            else:
                out.append(MinerResponse(uid, query, str((reply.get("result") or {}).get("response", ""))))
        return out

    def score_responses(self, responses: Sequence[MinerResponse], *, normalize: bool = True) -> list[WeightedScore]:
        raw = [(r.uid, 0.0 if r.error is not None or not r.response else float(self._scorer.score(r.query, r.response)),
                r.response) for r in responses]
        total = sum(s for _, s, _ in raw)
        def weight(s: float) -> float:
            if not normalize:
                return s
            return s / total if total > 0 else 1.0 / max(len(raw), 1)
        return [WeightedScore(u, s, weight(s), resp) for u, s, resp in raw]

    def query_and_score(self, query: str, *, normalize: bool = True) -> list[WeightedScore]:
        return self.score_responses(self.query_all(query), normalize=normalize)


def cohort_consensus_score(query: str, response: str, *, peer_responses: Sequence[str]) -> float:
    """Fraction of peer responses sharing at least one whitespace token with ``response``."""
    del query
    mine = set(response.lower().split())
    if not mine or not peer_responses:
        return 0.0
    return sum(1 for p in peer_responses if mine & set(p.lower().split())) / len(peer_responses)


def aggregate_cohort_scores(raw_scores: Sequence[float], *, mode: str = "mean") -> float:
    if not raw_scores:
        return 0.0
    fns = {"mean": statistics.fmean, "median": statistics.median, "max": max, "min": min}
    if mode not in fns:
        raise ValueError(f"unknown mode {mode!r}; use mean / median / max / min")
    return float(fns[mode](raw_scores))


__all__ = ["BittensorMinerServer", "BittensorValidatorClient", "MinerHandler", "MinerInfo", "MinerResponse",
           "ValidatorScorer", "WeightedScore", "aggregate_cohort_scores", "cohort_consensus_score"]

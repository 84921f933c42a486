"""Parallelism: expert parallelism (dispatch/combine), data-parallel gradient sync, and
the distributed-training building blocks of the reference (ZeRO planner, DiLoCo/NoLoCo,
gradient compression, verification, reputation, decentralised rounds)."""

from saint_llm_b200.parallel.ep import (
    DispatchPlan,
    combine_outputs_by_expert,
    dispatch_tokens_by_expert,
    setup_expert_parallel,
)

__all__ = ["DispatchPlan", "combine_outputs_by_expert", "dispatch_tokens_by_expert", "setup_expert_parallel"]

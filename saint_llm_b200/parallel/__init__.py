"""Parallelism: expert parallelism (NCCL baseline and the peer-memory kernels of
``ep_p2p``), data-parallel gradient sync, tensor parallelism for attention (``tp``) and its
composition with EP and hybrid ZeRO (``tp_ep``), full state dicts of sharded models
(``state``), two-stage context parallelism (``cp``), 1F1B pipeline parallelism (``pipeline``), and
the distributed-training building blocks of the reference (ZeRO planner and runtime,
DiLoCo/NoLoCo, gradient compression, verification, reputation, decentralised rounds,
miner/validator protocol, FSDP2 wrapping)."""

from saint_llm_b200.parallel.compression import (
    CompressedGradient,
    SparseLoCoBloom,
    TopKWithResidualCompressor,
    bloom_size_for,
    decompress,
    sparse_loco_compress,
    top_k_compression,
)
from saint_llm_b200.parallel.ep import (
    DispatchPlan,
    combine_outputs_by_expert,
    dispatch_tokens_by_expert,
    setup_expert_parallel,
)
from saint_llm_b200.parallel.local_sgd import (
    AllReduceReducer,
    DiLoCo,
    DiLoCoConfig,
    IdentityReducer,
    NoLoCo,
    NoLoCoConfig,
    RingAllReduceSimulator,
    ring_all_reduce,
)
from saint_llm_b200.parallel.state import gather_full_state_dict, load_full_state_dict
from saint_llm_b200.parallel.tp_ep import TPEPLayout, parallel_decode, setup_tp_ep, shard_for_inference
from saint_llm_b200.parallel.trust import (
    DecentralizedTrainingRound,
    GradientVerifier,
    PeerReputationConfig,
    PeerReputationTracker,
    PeerSubmission,
    reputation_weighted_reduce,
)
from saint_llm_b200.parallel.zero import (
    BucketAssignment,
    ZeroOptimizerSync,
    hybrid_zero_assign,
    pack_buckets_by_cost,
)

__all__ = ["AllReduceReducer", "BucketAssignment", "CompressedGradient", "DecentralizedTrainingRound", "DiLoCo",
           "DiLoCoConfig", "DispatchPlan", "GradientVerifier", "IdentityReducer", "NoLoCo", "NoLoCoConfig",
           "PeerReputationConfig", "PeerReputationTracker", "PeerSubmission", "RingAllReduceSimulator",
           "SparseLoCoBloom", "TPEPLayout", "TopKWithResidualCompressor", "ZeroOptimizerSync", "bloom_size_for",
           "combine_outputs_by_expert", "decompress", "dispatch_tokens_by_expert", "gather_full_state_dict",
           "hybrid_zero_assign", "load_full_state_dict", "pack_buckets_by_cost", "parallel_decode",
           "reputation_weighted_reduce", "ring_all_reduce", "setup_expert_parallel", "setup_tp_ep",
           "shard_for_inference", "sparse_loco_compress", "top_k_compression"]

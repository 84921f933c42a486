"""Post-training: GRPO family (GRPO / GSPO / DAPO / Dr.GRPO, GTPO, Tree-GRPO, Critique-GRPO),
rollouts, SFT, on-policy distillation, generative reward models, process reward models,
caption rewards, multimodal GRPO/SFT and the specialist pipeline."""

from saint_llm_b200.posttrain.caption_rewards import (
    PerExampleCaptionRewardFn,
    composite_caption_reward,
    constant_reward,
    length_target_reward,
    unigram_overlap_reward,
)
from saint_llm_b200.posttrain.critique import (
    CritiqueGRPOConfig,
    CritiqueRequest,
    collect_critique_requests,
    make_critique_prompt,
    make_refinement_prompt,
    needs_critique_mask,
)
from saint_llm_b200.posttrain.grm import GRMConfig, GRMRewardFn, binary_grm_config, judge_completion, likert_grm_config
from saint_llm_b200.posttrain.grpo import (
    GRPOConfig,
    RolloutBatch,
    compute_group_advantage,
    dynamic_sampling_mask,
    gather_token_logprobs,
    grpo_loss,
    grpo_loss_from_logprobs,
    overlong_reward_shape,
    policy_token_logprobs,
)
from saint_llm_b200.posttrain.gtpo import GTPOConfig, entropy_weight, gtpo_loss, per_token_entropy
from saint_llm_b200.posttrain.multimodal_grpo import (
    MultimodalRolloutBatch,
    build_multimodal_rollout_batch,
    multimodal_grpo_train_step,
)
from saint_llm_b200.posttrain.opd import OPDConfig, aggregate_teacher_logits, opd_kl_loss, opd_step
from saint_llm_b200.posttrain.rollout import RolloutGenConfig, decode_rollouts_for_reward, generate_grpo_rollouts
from saint_llm_b200.posttrain.sft import (
    JsonlSFTDataset,
    SFTExample,
    SFTPackedBatch,
    encode_sft,
    multimodal_sft_loss,
    multimodal_sft_step,
    pack_sft_examples,
    pack_sft_into_batch,
    sft_cross_entropy,
    sft_loss,
)
from saint_llm_b200.posttrain.specialist import RLStepOutput, SFTStepOutput, SpecialistPipeline
from saint_llm_b200.posttrain.think_prm import (
    StepRewardHead,
    ThinkPRMConfig,
    compute_step_rewards,
    find_step_boundaries,
    gather_step_logits,
    gather_step_scores,
    prm_filter_mask,
    step_prm_loss,
)
from saint_llm_b200.posttrain.trainer import GRPOTrainerStep, RewardFn, build_rollout_batch, grpo_train_step, score_rollouts
from saint_llm_b200.posttrain.tree_grpo import (
    TreeGRPOTrainerStep,
    TreeRolloutBatch,
    build_tree_rollout_batch,
    compute_tree_advantage,
    tree_dynamic_sampling_mask,
    tree_grpo_loss,
    tree_grpo_train_step,
)

__all__ = [n for n in dir() if not n.startswith("_")]

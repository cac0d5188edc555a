"""Long-context math GRPO on MiniCPM5-2B at 128k (reference ``recipe/math_grpo_minicpm5_2b.py``).

Trainer: context parallel CP4 x DP2 over 8 cards (CP4 x DP1 on the 4-card variant), full activation
checkpointing, rollout-side old log-probs with truncated importance sampling.  Rollout: S9 math prompts,
the "2.6 math" reshaped advantage (overlong soft penalty + length reward), zero-variance groups dropped,
no pacing window.  :func:`build` serves both node sizes.
"""

from __future__ import annotations

import os

from meshy_b200.config import GlobalCheckpointConfig, SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

SEQ_LEN = 131072
MAX_NEW_TOKENS = 126976
GROUP_SIZE = 8
CP = 4


def build(ngpus: int = 8, rollout_batch: int = 256, batch_size: int = 512):
    ngpus = int(os.environ.get("XRL_NGPUS", ngpus))
    if ngpus % CP:
        raise ValueError(f"{ngpus} cards do not divide into CP{CP} groups")
    tc = TrainerConfig(model_name="minicpm5", model_flavor="2B", seq_len=SEQ_LEN, lr=1e-6, weight_decay=0.0,
                       eps=1e-8, max_norm=1.0, dtype="bfloat16", activation_checkpoint_mode="full",
                       dp_shard_degree=1, dp_replicate_degree=ngpus // CP, cp_degree=CP, enable_checkpoint=True,
                       dump_folder="./outputs/math_grpo_minicpm5_2b")
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="padded", old_logprobs_source="rollout", use_tis=True,
                             ppo_clip_eps_high=0.28)
    return grpo_graph(
        model="minicpm5:2B", model_path=local_model_path(), trainer_config=tc, trainer_params=tp,
        batch_size=batch_size, rollout_batch=rollout_batch, group_size=GROUP_SIZE,
        dataset="meshy_b200.dataset.math:S9Math", dataset_kwargs={"seed": 42},
        reward="meshy_b200.dataset.math:S9Math.reward", sampling=SamplingParams(max_new_tokens=MAX_NEW_TOKENS),
        n_infer=ngpus, pacing_window=None, async_max_running_request=1024, filter_zero_std_groups=True,
        advantage="meshy_b200.advantage:_2_6_math_reshaped_advantage",
        checkpoint=GlobalCheckpointConfig(enabled=True, interval=10),
        server_args={"context_length": SEQ_LEN},
        rollout_extra={"advantage_kwargs": {"rollout_max_response_len": MAX_NEW_TOKENS, "overlong_buffer_len": 25395,
                                            "overlong_penalty_factor": 1.0, "length_reward_weight": 0.2,
                                            "length_reward_min_spread": 8000,
                                            "length_reward_budget_floor": 10000}})


SERVICE_GROUPS, COLOCATIONS = build()


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

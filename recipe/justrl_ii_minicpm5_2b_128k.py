"""PPO with a VAPO-GAE critic on MiniCPM5-2B at 128k context, one 8-card node
(reference ``recipe/justrl_ii_minicpm5_2b_128k.py``).

All 8 cards are shared serially by inference (FALLBACK), the critic and the actor trainer (both ON_DEMAND).
Actor and critic are CP4 x DP2 replicas (head-tail sharded 128k sequences, full activation checkpointing).

* batch 60 prompts x 8, 126976-token response cap, T=1.0 / top_p=1.0;
* clip-higher 0.2 / 0.28, TIS over [0.5, 5.0], no KL / reference model;
* DAPO overlong soft penalty (buffer 25395, factor 1.0) as reward shaping; the raw reward is kept;
* dynamic sampling: zero-variance groups dropped, 2x oversampling to refill the window;
* positive LM loss 0.1 on shaped-reward > 0.5 samples, weighted by raw-group difficulty;
* critic cold start (``XRL_COLD_START_WINDOWS``, default 20) with the actor frozen;
* global checkpoints every 10 windows, 2 retained.

``XRL_NGPUS`` rescales the replicas (a multiple of 4); the 32-card two-group layout is
``recipe.justrl_ii_minicpm5_2b_128k_32gpu``.
"""

from __future__ import annotations

import os

from meshy_b200.config import (CriticServiceConfig, SamplingParams, TrainerConfig,
                               TrainerParamsConfig)
from meshy_b200.recipe_lib import checkpoint_from_env, grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

SEQ_LEN = 131072
MAX_NEW_TOKENS = 126976
OVERLONG_BUFFER_LEN = 25395
OVERLONG_PENALTY_FACTOR = 1.0
ROLLOUT_BATCH = 60
GROUP_SIZE = 8
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
CP = 4


def trainer_config(folder: str, ngpus: int) -> TrainerConfig:
    return TrainerConfig(model_name="minicpm5", model_flavor="2B", seq_len=SEQ_LEN, lr=1e-6, weight_decay=0.0,
                         eps=1e-8, max_norm=1.0, lr_decay_ratio=None, dtype="bfloat16",
                         activation_checkpoint_mode="full", dp_shard_degree=1, dp_replicate_degree=ngpus // CP,
                         cp_degree=CP, dump_folder=folder)


def trainer_params() -> TrainerParamsConfig:
    return TrainerParamsConfig(mini_batch_size=4, batch_layout="padded", old_logprobs_source="train", use_tis=True,
                               tis_ratio_min=0.5, tis_ratio_max=5.0, ppo_clip_eps_low=0.2, ppo_clip_eps_high=0.28,
                               positive_lm_loss_coef=0.1, enable_gae=True, gae_gamma=1.0, gae_alpha=1.5)


def build(ngpus: int = 8, critic_colocate: bool = True, n_critic: int | None = None):
    cold = int(os.environ.get("XRL_COLD_START_WINDOWS", "20"))
    score_batch = int(os.environ.get("XRL_CRITIC_SCORE_BATCH", str(BATCH_SIZE)))
    ckpt = checkpoint_from_env(interval=10, keep_latest_k=3)  # XRL_CHECKPOINT / _INTERVAL / _KEEP
    path = local_model_path()
    n_critic = n_critic or ngpus
    if ngpus % CP or n_critic % CP:
        raise ValueError(f"card counts must be multiples of CP{CP}")
    return grpo_graph(
        model="minicpm5:2B", model_path=path, trainer_config=trainer_config("./outputs/justrl_ii_128k/actor", ngpus),
        trainer_params=trainer_params(), batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
        dataset="meshy_b200.dataset.math:S9Math", dataset_kwargs={"seed": 42},
        reward="meshy_b200.dataset.math:S9Math.reward",
        reward_shaping="meshy_b200.reward:soft_overlong_penalty",
        reward_shaping_kwargs={"max_response_len": MAX_NEW_TOKENS, "buffer_len": OVERLONG_BUFFER_LEN,
                               "penalty_factor": OVERLONG_PENALTY_FACTOR},
        filter_zero_std_groups=True, oversample_factor=2.0,
        sampling=SamplingParams(max_new_tokens=MAX_NEW_TOKENS), n_infer=ngpus, pacing_window=1,
        server_args={"context_length": SEQ_LEN}, checkpoint=ckpt, critic_colocate=critic_colocate,
        n_critic=n_critic, rollout_extra={"publish_positive_lm_weights": True},
        critic=CriticServiceConfig(model_path=path,
                                   trainer_config=trainer_config("./outputs/justrl_ii_128k/critic", n_critic),
                                   score_batch_size=score_batch, publish_mode="values", lr=5e-6,
                                   cold_start_windows=cold, checkpoint=ckpt))


SERVICE_GROUPS, COLOCATIONS = build(int(os.environ.get("XRL_NGPUS", "8")))


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

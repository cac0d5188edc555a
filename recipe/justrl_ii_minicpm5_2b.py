"""PPO with an independent VAPO-GAE critic on MiniCPM5-2B, one 8-card node
(reference ``recipe/justrl_ii_minicpm5_2b.py``).

Cards 0-3: inference replicas time-sharing with the 4-card actor trainer; cards 4-7: a dedicated 4-card
critic (no arbitration, so critic scoring overlaps generation).  The rollout computes no advantage: the
critic scores each window with its pre-update weights, publishes ``values`` and the trainer turns them into
per-token GAE advantages.  For ``XRL_COLD_START_WINDOWS`` windows the critic trains alone and the actor
stays frozen.  Global checkpoints of actor, critic and rollout cursor land together.
"""

from __future__ import annotations

import os

from meshy_b200.config import (CriticServiceConfig, SamplingParams, TrainerConfig,
                               TrainerParamsConfig)
from meshy_b200.recipe_lib import checkpoint_from_env, grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

MODEL_PATH = local_model_path()
NUM_INFERENCE_ENGINES = 4
NUM_CRITIC_CARDS = 4
ROLLOUT_BATCH = 16
GROUP_SIZE = 8
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
SEQ_LEN = 4096
MAX_NEW_TOKENS = 1024
COLD_START_WINDOWS = int(os.environ.get("XRL_COLD_START_WINDOWS", "2"))
CHECKPOINT = checkpoint_from_env(interval=10, keep_latest_k=3)  # XRL_CHECKPOINT / _INTERVAL / _KEEP


def _tc(folder: str, ckpt: str = "selective", shard: int = NUM_INFERENCE_ENGINES) -> TrainerConfig:
    return TrainerConfig(model_name="minicpm5", model_flavor="2B", seq_len=SEQ_LEN, lr=1e-6, weight_decay=0.0,
                         eps=1e-8, max_norm=1.0, dtype="bfloat16", dp_shard_degree=-1, dp_replicate_degree=1,
                         activation_checkpoint_mode=ckpt, dump_folder=folder)


SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model="minicpm5:2B", model_path=MODEL_PATH, trainer_config=_tc("./outputs/justrl_ii_minicpm5_2b/actor"),
    trainer_params=TrainerParamsConfig(mini_batch_size=8, batch_layout="packed", max_tokens_per_micro=32768,
                                       old_logprobs_source="train", enable_gae=True, gae_gamma=1.0, gae_alpha=1.5),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(max_new_tokens=MAX_NEW_TOKENS), n_infer=NUM_INFERENCE_ENGINES, pacing_window=1,
    checkpoint=CHECKPOINT, critic_colocate=False, n_critic=NUM_CRITIC_CARDS,
    critic=CriticServiceConfig(model_path=MODEL_PATH,
                               trainer_config=_tc("./outputs/justrl_ii_minicpm5_2b/critic", "full"),
                               score_batch_size=BATCH_SIZE, publish_mode="values", max_tokens_per_micro=32768,
                               lr=5e-6, cold_start_windows=COLD_START_WINDOWS, checkpoint=CHECKPOINT))


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

"""Writes a verbose ``trajectories.jsonl`` fixture for the offline critic tools
(reference ``recipe/critic_traj_dump.py``).

The 4-card colocated JustRL-MiniCPM5-2B graph shrunk to a fixture: 16 prompts x 4 rollouts per window,
512-token responses, a bounded prompt set (``XRL_DUMP_BATCHES`` windows), and token-level trajectory rows
(``verbose_trajectory_log=True``) that ``meshy_b200.backend.critic.data`` and
``meshy_b200.bench.train_only --trajectories`` read back.
"""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

NUM_INFERENCE_ENGINES = 4
ROLLOUT_BATCH = 16
GROUP_SIZE = 4
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
MAX_NEW_TOKENS = 512
SEQ_LEN = 2048
DUMP_BATCHES = int(os.environ.get("XRL_DUMP_BATCHES", "4"))

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model="minicpm5:2B", model_path=local_model_path(),
    trainer_config=TrainerConfig(model_name="minicpm5", model_flavor="2B", seq_len=SEQ_LEN, lr=1e-6,
                                 weight_decay=0.0, dtype="bfloat16", dp_shard_degree=1,
                                 dp_replicate_degree=NUM_INFERENCE_ENGINES, dump_folder="./outputs/critic_traj_dump"),
    trainer_params=TrainerParamsConfig(mini_batch_size=8, batch_layout="packed", max_tokens_per_micro=16384,
                                       old_logprobs_source="train"),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42, "limit": DUMP_BATCHES * ROLLOUT_BATCH},
    reward="meshy_b200.dataset.math:MATH.reward", sampling=SamplingParams(max_new_tokens=MAX_NEW_TOKENS),
    n_infer=NUM_INFERENCE_ENGINES, pacing_window=1, rollout_extra={"verbose_trajectory_log": True})


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

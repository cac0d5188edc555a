"""JustRL on MiniCPM5-2B, one 8-card node, colocated (reference ``recipe/justrl_minicpm5_2b.py``).

8 single-card inference replicas and an 8-way data-parallel trainer time-share the cards; MATH prompts,
256 x 8 rollouts per window, 15360-token responses, checkpoints every 10 windows.  ``MINICPM5_LOCAL_PATH``
names the checkpoint (random init of the architecture when unset); ``XRL_NGPUS`` scales the node.
:func:`build` also serves the 1B and 4-card variants.
"""

from __future__ import annotations

import os

from meshy_b200.config import GlobalCheckpointConfig, SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

GROUP_SIZE = 8
NUM_EPOCHS = 8


def build(flavor: str = "2B", ngpus: int | None = None):
    ngpus = ngpus or int(os.environ.get("XRL_NGPUS", "8"))
    rollout_batch = int(os.environ.get("XRL_ROLLOUT_BATCH", "256"))
    tc = TrainerConfig(model_name="minicpm5", model_flavor=flavor, seq_len=16384, lr=1e-6, weight_decay=0.0,
                       eps=1e-8, max_norm=1.0, dtype="bfloat16", dp_shard_degree=1, dp_replicate_degree=ngpus,
                       enable_checkpoint=True, dump_folder=f"./outputs/justrl_minicpm5_{flavor.lower()}")
    return grpo_graph(
        model=f"minicpm5:{flavor}", model_path=local_model_path(), trainer_config=tc,
        trainer_params=TrainerParamsConfig(mini_batch_size=8, batch_layout="packed", max_tokens_per_micro=32768,
                                           old_logprobs_source="train"),
        batch_size=rollout_batch * GROUP_SIZE, rollout_batch=rollout_batch, group_size=GROUP_SIZE,
        dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42},
        reward="meshy_b200.dataset.math:MATH.reward", sampling=SamplingParams(max_new_tokens=15360), n_infer=ngpus,
        pacing_window=1, num_epochs=NUM_EPOCHS, checkpoint=GlobalCheckpointConfig(enabled=True, interval=10),
        rollout_extra={"verbose_trajectory_log": os.environ.get("XRL_VERBOSE_TRAJ", "0") == "1"})


SERVICE_GROUPS, COLOCATIONS = build()


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

"""JustRL on Qwen3-30B-A3B (reference ``recipe/justrl_qwen3_30b_a3b.py``).

Trainer: 8 cards with expert parallelism EP8 (each rank owns 16 of the 128 experts; dense weights
data-parallel) -- new relative to the reference, whose trainer has no EP.  Inference: the reference needs
TP8 + EP8 because 60 GB of bf16 weights do not fit one 80 GB card; on a 180 GB B200 they do, so each card
runs a full single-card replica (replica-level data parallelism of inference instead of TP)."""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph
from meshy_b200.service.ignite import Ignitor

NGPUS = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "32"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "8"))

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model="qwen3:30B-A3B", model_path=os.environ.get("MODEL_PATH") or None,
    trainer_config=TrainerConfig(model_name="qwen3", model_flavor="30B-A3B", seq_len=16384, lr=1e-6,
                                 weight_decay=0.1, dtype="bfloat16", dp_shard_degree=1, dp_replicate_degree=NGPUS,
                                 ep_degree=NGPUS, activation_checkpoint_mode="full"),
    trainer_params=TrainerParamsConfig(mini_batch_size=1, batch_layout="packed", max_tokens_per_micro=16384,
                                       old_logprobs_source="train"),
    batch_size=ROLLOUT_BATCH * GROUP_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(max_new_tokens=int(os.environ.get("XRL_MAX_NEW_TOKENS", "15360"))), n_infer=NGPUS,
    server_args={"mem_fraction_static": 0.7}, pacing_window=1)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

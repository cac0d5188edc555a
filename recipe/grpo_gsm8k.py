"""GRPO on GSM8K (reference ``recipe/grpo_gsm8k.py``): a small, env-tunable recipe.

``XRL_MODEL`` (registry ``name:flavor``, default ``qwen2_5:1.5B``), ``XRL_NGPUS``, ``XRL_ROLLOUT_BATCH``,
``XRL_GROUP_SIZE``, ``XRL_MAX_NEW_TOKENS``, ``XRL_SEQ_LEN``; data from ``GSM8K_DATASET_PATH``."""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph
from meshy_b200.service.ignite import Ignitor

MODEL = os.environ.get("XRL_MODEL", "qwen2_5:1.5B")
NGPUS = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "64"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "8"))
SEQ_LEN = int(os.environ.get("XRL_SEQ_LEN", "2048"))
_name, _flavor = MODEL.split(":")

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=MODEL, model_path=os.environ.get("MODEL_PATH") or None,
    trainer_config=TrainerConfig(model_name=_name, model_flavor=_flavor, seq_len=SEQ_LEN, lr=1e-6, weight_decay=0.0,
                                 dtype="bfloat16", dp_shard_degree=1, dp_replicate_degree=NGPUS),
    trainer_params=TrainerParamsConfig(mini_batch_size=8, batch_layout="packed", max_tokens_per_micro=16384,
                                       old_logprobs_source="train"),
    batch_size=ROLLOUT_BATCH * GROUP_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:GSM8K", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:GSM8K.reward",
    sampling=SamplingParams(max_new_tokens=int(os.environ.get("XRL_MAX_NEW_TOKENS", "1024"))), n_infer=NGPUS)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

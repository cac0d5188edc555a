"""GRPO on GSM8K with Qwen3-8B (reference ``recipe/grpo_gsm8k_qwen3_8b.py``).

8 single-card inference replicas colocated with one 8-card trainer whose optimiser state is sharded over
the DP ranks (``dp_shard_degree=-1``: the fused NVLink reduce-scatter / AdamW / all-gather keeps each rank's
fp32 moments for its shard only; bf16 weights stay resident, 16 GB, well inside a B200's 180 GB)."""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, model_from_env
from meshy_b200.service.ignite import Ignitor

# the reference's variables: XRL_MODEL (checkpoint dir; random init without a local copy), XRL_MODEL_NAME /
# XRL_MODEL_FLAVOR, XRL_NGPUS, XRL_SEQ_LEN, XRL_MAX_NEW_TOKENS, XRL_ROLLOUT_BATCH, XRL_GROUP_SIZE, XRL_STEPS,
# XRL_LR, XRL_EPOCHS (the sequence defaults follow the benchmark configuration: 4k tokens, responses to 2k)
NAME, FLAVOR, MODEL_PATH = model_from_env("qwen3", "8B")
NGPUS = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "32"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "8"))
SEQ_LEN = int(os.environ.get("XRL_SEQ_LEN", "4096"))

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=f"{NAME}:{FLAVOR}", model_path=MODEL_PATH,
    trainer_config=TrainerConfig(model_name=NAME, model_flavor=FLAVOR, seq_len=SEQ_LEN,
                                 steps=int(os.environ.get("XRL_STEPS", "1000")),
                                 lr=float(os.environ.get("XRL_LR", "1e-6")), weight_decay=0.1,
                                 dtype="bfloat16", dp_shard_degree=-1, dp_replicate_degree=1,
                                 dump_folder="./outputs/grpo_gsm8k_qwen3_8b"),
    trainer_params=TrainerParamsConfig(mini_batch_size=1, batch_layout="packed", max_tokens_per_micro=16384,
                                       old_logprobs_source="train"),
    batch_size=ROLLOUT_BATCH * GROUP_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:GSM8K", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:GSM8K.reward",
    sampling=SamplingParams(max_new_tokens=int(os.environ.get("XRL_MAX_NEW_TOKENS", "2048"))), n_infer=NGPUS,
    pacing_window=1, num_epochs=int(os.environ.get("XRL_EPOCHS", "1")))


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

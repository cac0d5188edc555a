"""GRPO on GSM8K (reference ``recipe/grpo_gsm8k.py``): a small, environment-tunable recipe that drives
single-card smoke runs and multi-card runs alike.

Variables (the reference's names and defaults): ``XRL_MODEL`` (checkpoint directory, default
``Qwen/Qwen3-1.7B``: random-init weights when no local copy exists), ``XRL_MODEL_NAME`` / ``XRL_MODEL_FLAVOR``
(architecture, ``qwen3`` / ``1.7B``), ``XRL_NGPUS`` (1), ``XRL_TOPOLOGY`` (``colocate``: inference and trainer
share every card; ``disaggregate``: inference on ``XRL_NGPUS - XRL_TRAIN_GPUS`` cards, the trainer on
``XRL_TRAIN_GPUS``, default half), ``XRL_SEQ_LEN`` (2048), ``XRL_MAX_NEW_TOKENS`` (1024), ``XRL_ROLLOUT_BATCH``
(4 prompts), ``XRL_GROUP_SIZE`` (4), ``XRL_STEPS`` (1000, the LR schedule's horizon), ``XRL_LR`` (1e-6),
``XRL_EPOCHS`` (1). Data from ``GSM8K_DATASET_PATH`` (JSONL).

Inference runs one single-card replica per card; ``XRL_INFER_TP`` groups the cards into tensor-parallel
replicas instead (the reference's colocated layout is one replica over all ``XRL_NGPUS`` cards).
"""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, model_from_env
from meshy_b200.service.ignite import Ignitor

NAME, FLAVOR, MODEL_PATH = model_from_env("qwen3", "1.7B")
NGPUS = int(os.environ.get("XRL_NGPUS", "1"))
TOPOLOGY = os.environ.get("XRL_TOPOLOGY", "colocate")
SEQ_LEN = int(os.environ.get("XRL_SEQ_LEN", "2048"))
MAX_NEW_TOKENS = int(os.environ.get("XRL_MAX_NEW_TOKENS", "1024"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "4"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "4"))
INFER_TP = int(os.environ.get("XRL_INFER_TP", "1"))


def build():
    if TOPOLOGY == "colocate":
        n_infer = n_train = NGPUS
    elif TOPOLOGY == "disaggregate":
        if NGPUS < 2:
            raise ValueError("disaggregate topology needs XRL_NGPUS >= 2")
        n_train = int(os.environ.get("XRL_TRAIN_GPUS", str(max(1, NGPUS // 2))))
        n_infer = NGPUS - n_train
        if n_infer < 1:
            raise ValueError("disaggregate needs at least 1 inference card")
    else:
        raise ValueError(f"unknown XRL_TOPOLOGY={TOPOLOGY!r} (use 'colocate' or 'disaggregate')")
    return grpo_graph(
        model=f"{NAME}:{FLAVOR}", model_path=MODEL_PATH,
        trainer_config=TrainerConfig(model_name=NAME, model_flavor=FLAVOR, seq_len=SEQ_LEN,
                                     steps=int(os.environ.get("XRL_STEPS", "1000")),
                                     lr=float(os.environ.get("XRL_LR", "1e-6")), dtype="bfloat16",
                                     dp_shard_degree=1, dp_replicate_degree=n_train,
                                     dump_folder="./outputs/grpo_gsm8k"),
        trainer_params=TrainerParamsConfig(mini_batch_size=1, batch_layout="packed", max_tokens_per_micro=16384,
                                           ppo_clip_eps_low=0.2, ppo_clip_eps_high=0.2,
                                           old_logprobs_source="rollout"),
        batch_size=ROLLOUT_BATCH * GROUP_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
        dataset="meshy_b200.dataset.math:GSM8K", dataset_kwargs={"seed": 42},
        reward="meshy_b200.dataset.math:GSM8K.reward",
        sampling=SamplingParams(temperature=1.0, top_p=1.0, top_k=-1, max_new_tokens=MAX_NEW_TOKENS),
        n_infer=n_infer, n_train=n_train, colocate=TOPOLOGY == "colocate", pacing_window=1,
        num_epochs=int(os.environ.get("XRL_EPOCHS", "1")), infer_tp=INFER_TP)


SERVICE_GROUPS, COLOCATIONS = build()


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

"""JustRL: GRPO for the DeepSeek-R1-Distill-Qwen-1.5B architecture on DAPO-Math-17k (reference ``recipe/justrl.py``).

8 cards, colocated: 8 single-card inference replicas and one DDP-8 trainer hand the cards back and forth
through the colocation ring; lock-step pacing (``pacing_window=1``).  256 prompts x 8 = 2048 samples per
step, 15360-token responses, seq_len 16384.  Weights: ``MODEL_PATH`` (an HF checkpoint dir) or random init.
Data: ``MATH_DATASET_PATH`` (JSONL with ``prompt``/``answer``).

    python -m meshy_b200.launch --recipe recipe.justrl
"""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph
from meshy_b200.service.ignite import Ignitor

MODEL = "qwen2_5_math:R1-Distill-1.5B"
MODEL_PATH = os.environ.get("MODEL_PATH") or None
NGPUS = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "256"))
GROUP_SIZE = 8
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
NUM_EPOCHS = 8


def trainer_config() -> TrainerConfig:
    return TrainerConfig(model_name="qwen2_5_math", model_flavor="R1-Distill-1.5B", seq_len=16384, lr=1e-6,
                         weight_decay=0.1, warmup_steps=0, max_norm=1.0, steps=3000, dtype="bfloat16",
                         dp_shard_degree=1, dp_replicate_degree=NGPUS)


def trainer_params() -> TrainerParamsConfig:
    return TrainerParamsConfig(mini_batch_size=8, micro_batch_size=1, ppo_clip_eps_low=0.2, ppo_clip_eps_high=0.28,
                               old_logprobs_source="train", batch_layout="packed", max_tokens_per_micro=32768)


SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=MODEL, model_path=MODEL_PATH, trainer_config=trainer_config(), trainer_params=trainer_params(),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(temperature=1.0, top_p=1.0, top_k=-1, max_new_tokens=15360), n_infer=NGPUS,
    server_args={"mem_fraction_static": 0.6, "enable_memory_saver": True}, pacing_window=1, num_epochs=NUM_EPOCHS)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

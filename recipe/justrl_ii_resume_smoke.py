"""Kill-and-resume smoke of the JustRL-II graph (reference ``recipe/justrl_ii_resume_smoke.py``).

The same four services and ring as JustRL-II (inference FALLBACK, critic and actor trainer ON_DEMAND on all
cards, rollout on CPU), shrunk so a global checkpoint lands every window: R1-Distill-Qwen-1.5B, 4 prompts
x 4 rollouts, 256-token responses, two critic cold-start windows (a kill can land on either side of the
critic -> trainer hand-off), ``XRL_SMOKE_BATCHES`` prompt batches.  The critic publishes finished
advantages (``publish_mode="advantage"``).

    python -m meshy_b200.launch --recipe recipe.justrl_ii_resume_smoke --runtime-dir RUN
    # interrupt it after a few checkpoints, then
    python -m meshy_b200.launch --recipe recipe.justrl_ii_resume_smoke --runtime-dir RUN --resume

On resume every role restores the newest step all of them committed: trainer weights and optimiser, the
critic's value net and optimiser, the rollout's data cursor and the generation gate stream.
"""

from __future__ import annotations

import os

from meshy_b200.config import (CriticServiceConfig, GlobalCheckpointConfig, SamplingParams, TrainerConfig,
                               TrainerParamsConfig)
from meshy_b200.recipe_lib import grpo_graph, local_model_path
from meshy_b200.service.ignite import Ignitor

MODEL_PATH = local_model_path("XRL_MODEL")
NUM_INFERENCE_ENGINES = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = 4
GROUP_SIZE = 4
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
SEQ_LEN = 1024
MAX_NEW_TOKENS = 256
COLD_START_WINDOWS = int(os.environ.get("XRL_COLD_START_WINDOWS", "2"))
CHECKPOINT = GlobalCheckpointConfig(enabled=True, interval=int(os.environ.get("XRL_CHECKPOINT_INTERVAL", "1")),
                                    keep_latest_k=int(os.environ.get("XRL_CHECKPOINT_KEEP", "2")))
NUM_PROMPT_BATCHES = int(os.environ.get("XRL_SMOKE_BATCHES", "40"))


def _tc(folder: str) -> TrainerConfig:
    return TrainerConfig(model_name="qwen2_5_math", model_flavor="R1-Distill-1.5B", seq_len=SEQ_LEN, lr=1e-6,
                         weight_decay=0.0, dtype="bfloat16", dp_shard_degree=-1, dp_replicate_degree=1,
                         activation_checkpoint_mode="full", dump_folder=folder)


SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model="qwen2_5_math:R1-Distill-1.5B", model_path=MODEL_PATH, trainer_config=_tc("./outputs/resume_smoke/actor"),
    trainer_params=TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=8192,
                                       old_logprobs_source="train"),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH",
    dataset_kwargs={"seed": 42, "limit": NUM_PROMPT_BATCHES * ROLLOUT_BATCH},
    reward="meshy_b200.dataset.math:MATH.reward", sampling=SamplingParams(max_new_tokens=MAX_NEW_TOKENS),
    n_infer=NUM_INFERENCE_ENGINES, pacing_window=1, checkpoint=CHECKPOINT,
    critic=CriticServiceConfig(model_path=MODEL_PATH, trainer_config=_tc("./outputs/resume_smoke/critic"),
                               score_batch_size=BATCH_SIZE, publish_mode="advantage", lr=5e-6, warmup_steps=2,
                               cold_start_windows=COLD_START_WINDOWS, checkpoint=CHECKPOINT))


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

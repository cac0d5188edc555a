"""Critic-only cold start at 32k on MiniCPM5-2B-SFT (reference ``recipe/critic_coldstart_32k.py``).

6 inference cards generate; a dedicated 2-card CP2 critic fits its value net to the shaped returns and
never publishes (``cold_start_windows=-1``: the actor is absent, the generation gate paces the rollout).
Used to pre-train a critic before a JustRL-II run.  ``XRL_NUM_EPOCHS`` and ``XRL_CRITIC_SCORE_BATCH``
override the defaults.
"""

from __future__ import annotations

import os

from meshy_b200.config import (CriticServiceConfig, InferenceServiceConfig, RolloutServiceConfig, SamplingParams,
                               TrainerConfig)
from meshy_b200.recipe_lib import local_model_path
from meshy_b200.service.base import ServiceGroup
from meshy_b200.service.ignite import Ignitor

MODEL_PATH = local_model_path()
SEQ_LEN = 32768
MAX_NEW_TOKENS = 28672
NUM_INFERENCE_CARDS = 6
NUM_CRITIC_CARDS = 2
ROLLOUT_BATCH = 16
GROUP_SIZE = 8
NUM_EPOCHS = int(os.environ.get("XRL_NUM_EPOCHS", "100"))
CRITIC_SCORE_BATCH = int(os.environ.get("XRL_CRITIC_SCORE_BATCH", "64"))


def build_service_groups() -> list[ServiceGroup]:
    critic_tc = TrainerConfig(model_name="minicpm5", model_flavor="2B", seq_len=SEQ_LEN, lr=5e-6, weight_decay=0.0,
                              dtype="bfloat16", dp_shard_degree=1, dp_replicate_degree=1,
                              cp_degree=NUM_CRITIC_CARDS, activation_checkpoint_mode="full",
                              dump_folder="./outputs/critic_coldstart_32k/critic")
    # declaration order: inference on cards 0-5, critic on 6-7
    return [
        ServiceGroup(id="actor_infer", n_replicas=NUM_INFERENCE_CARDS, n_gpus_per_replica=1,
                     config=InferenceServiceConfig(model_path=MODEL_PATH,
                                                   server_args={"model": "minicpm5:2B", "context_length": SEQ_LEN})),
        ServiceGroup(id="critic", n_replicas=1, n_gpus_per_replica=NUM_CRITIC_CARDS, wait_until=["actor_infer"],
                     config=CriticServiceConfig(model_path=MODEL_PATH, trainer_config=critic_tc,
                                                score_batch_size=CRITIC_SCORE_BATCH, publish_mode="values",
                                                lr=5e-6, cold_start_windows=-1)),
        ServiceGroup(id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=["actor_infer", "critic"],
                     config=RolloutServiceConfig(
                         model_path=MODEL_PATH, dataset="meshy_b200.dataset.math:S9Math",
                         dataset_kwargs={"batch_size": ROLLOUT_BATCH, "seed": 42},
                         reward="meshy_b200.dataset.math:S9Math.reward",
                         sampling_params=SamplingParams(max_new_tokens=MAX_NEW_TOKENS).as_dict(),
                         group_size=GROUP_SIZE, num_epochs=NUM_EPOCHS, pacing_window=None,
                         external_advantage=True)),
    ]


SERVICE_GROUPS = build_service_groups()
COLOCATIONS: list = []


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

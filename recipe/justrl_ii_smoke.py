"""Smoke recipe of the PPO-with-critic service graph (JustRL-II shape) on a tiny Qwen3.

One card (CPU with ``XRL_DEVICE=cpu``) shared by three ring members --
inference (FALLBACK), critic and actor trainer (ON_DEMAND) -- plus the rollout
driver.  The critic cold-starts for one window (it trains alone and raises the
generation gate), then publishes ``values`` that the trainer turns into
VAPO-GAE advantages.

    XRL_DEVICE=cpu python -m meshy_b200.launch --recipe recipe.justrl_ii_smoke
"""

from __future__ import annotations

import os

from meshy_b200.config import (GAE_TRAINER_FIELDS, CriticServiceConfig, InferenceServiceConfig, RolloutServiceConfig,
                               SamplingParams, TrainerConfig, TrainerParamsConfig, TrainingServiceConfig)
from meshy_b200.service.base import ServiceGroup
from meshy_b200.service.colocation import ColocationRing, SchedulingMode
from meshy_b200.service.ignite import Ignitor

PROMPTS, GROUP = 2, 2
STEPS = int(os.environ.get("XRL_SMOKE_STEPS", "3"))
COLD = int(os.environ.get("XRL_SMOKE_COLD", "1"))


def _tc() -> TrainerConfig:
    return TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=512, lr=1e-5, weight_decay=0.0,
                         max_norm=1.0, steps=1000, dtype="bfloat16", dp_replicate_degree=1)


SERVICE_GROUPS = [
    ServiceGroup(id="actor_infer", n_replicas=1, n_gpus_per_replica=1,
                 config=InferenceServiceConfig(server_args={"model": "qwen3:debugmodel", "max_running_requests": 8,
                                                            "max_total_tokens": 4096, "context_length": 512})),
    ServiceGroup(id="critic", n_replicas=1, n_gpus_per_replica=1, colocate_with="actor_infer",
                 wait_until=["actor_infer"],
                 config=CriticServiceConfig(model_path=None, trainer_config=_tc(), score_batch_size=PROMPTS * GROUP,
                                            publish_mode="values", max_tokens_per_micro=2048, lr=1e-4, warmup_steps=1,
                                            cold_start_windows=COLD)),
    ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=1, colocate_with="actor_infer",
                 wait_until=["actor_infer", "critic"],
                 config=TrainingServiceConfig(
                     model_path=None, trainer_config=_tc(), batch_size=PROMPTS * GROUP, weight_sync_mode="disk",
                     trainer_params=TrainerParamsConfig(mini_batch_size=PROMPTS * GROUP, batch_layout="packed",
                                                        max_tokens_per_micro=2048, old_logprobs_source="train",
                                                        enable_gae=True, gae_gamma=1.0),
                     tq_fields=list(GAE_TRAINER_FIELDS), critic_cold_start_windows=COLD)),
    ServiceGroup(id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=["actor_train", "critic"],
                 config=RolloutServiceConfig(
                     model_path=None, dataset="meshy_b200.dataset.synthetic:SyntheticPrompts",
                     dataset_kwargs={"batch_size": PROMPTS, "n_prompts": PROMPTS * (STEPS + COLD), "vocab_size": 2048,
                                     "min_len": 8, "max_len": 16, "seed": 2},
                     reward="meshy_b200.dataset.synthetic:SyntheticPrompts.reward",
                     sampling_params=SamplingParams(max_new_tokens=16).as_dict(), group_size=GROUP,
                     poll_interval=0.2, pacing_window=1, external_advantage=True)),
]

COLOCATIONS = [ColocationRing(group_id="actor", ring=(("actor_infer", SchedulingMode.FALLBACK),
                                                      ("critic", SchedulingMode.ON_DEMAND),
                                                      ("actor_train", SchedulingMode.ON_DEMAND)))]


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

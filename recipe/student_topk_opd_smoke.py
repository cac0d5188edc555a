"""Smoke recipe of Top-K on-policy distillation on a tiny Qwen3 (one card, CPU with ``XRL_DEVICE=cpu``).

Inference (FALLBACK), a frozen teacher and the student trainer (both ON_DEMAND) share one card in a
ring; the teacher appends Top-K columns to every rollout row and the student trains on the forward KL.
"""

from __future__ import annotations

import os

from meshy_b200.config import (OPD_TRAINER_FIELDS, InferenceServiceConfig, OPDTeacherConfig, OPDTrainingConfig,
                               RolloutServiceConfig, SamplingParams, TrainerConfig, TrainerParamsConfig)
from meshy_b200.service.base import ServiceGroup
from meshy_b200.service.colocation import ColocationRing, SchedulingMode
from meshy_b200.service.ignite import Ignitor

PROMPTS, GROUP = 2, 2
STEPS = int(os.environ.get("XRL_SMOKE_STEPS", "2"))


def _tc() -> TrainerConfig:
    return TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=512, lr=1e-5, weight_decay=0.0,
                         max_norm=1.0, steps=1000, dtype="bfloat16", dp_replicate_degree=1)


SERVICE_GROUPS = [
    ServiceGroup(id="actor_infer", n_replicas=1, n_gpus_per_replica=1,
                 config=InferenceServiceConfig(server_args={"model": "qwen3:debugmodel", "max_running_requests": 8,
                                                            "max_total_tokens": 4096, "context_length": 512})),
    ServiceGroup(id="teacher", n_replicas=1, n_gpus_per_replica=1, colocate_with="actor_infer",
                 wait_until=["actor_infer"],
                 config=OPDTeacherConfig(model_path=None, trainer_config=_tc(), top_k=4, score_batch_size=PROMPTS * GROUP)),
    ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=1, colocate_with="actor_infer",
                 wait_until=["actor_infer", "teacher"],
                 config=OPDTrainingConfig(
                     model_path=None, trainer_config=_tc(), batch_size=PROMPTS * GROUP, weight_sync_mode="disk",
                     trainer_params=TrainerParamsConfig(mini_batch_size=PROMPTS * GROUP, batch_layout="packed",
                                                        max_tokens_per_micro=2048, old_logprobs_source="rollout"),
                     tq_fields=list(OPD_TRAINER_FIELDS))),
    ServiceGroup(id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=["actor_train", "teacher"],
                 config=RolloutServiceConfig(
                     model_path=None, dataset="meshy_b200.dataset.synthetic:SyntheticPrompts",
                     dataset_kwargs={"batch_size": PROMPTS, "n_prompts": PROMPTS * STEPS, "vocab_size": 2048,
                                     "min_len": 8, "max_len": 16, "seed": 3},
                     reward="meshy_b200.dataset.synthetic:SyntheticPrompts.reward",
                     sampling_params=SamplingParams(max_new_tokens=16).as_dict(), group_size=GROUP,
                     poll_interval=0.2, pacing_window=1)),
]

COLOCATIONS = [ColocationRing(group_id="actor", ring=(("actor_infer", SchedulingMode.FALLBACK),
                                                      ("teacher", SchedulingMode.ON_DEMAND),
                                                      ("actor_train", SchedulingMode.ON_DEMAND)))]


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

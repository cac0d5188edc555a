"""Top-K on-policy distillation: a Qwen3-1.7B student learns from a frozen Qwen3-8B teacher
(reference ``recipe/student_topk_opd.py``).

The student generates; the teacher scores every rollout row and appends its Top-K token ids and
log-probs; the student trains on the forward KL over those K tokens.  ``XRL_TOPOLOGY``:

* ``colocate`` (default): inference (FALLBACK), teacher and student (ON_DEMAND) time-share all cards;
* ``disaggregate``: ``XRL_TEACHER_GPUS`` teacher cards, the rest split between inference replicas and the
  student trainer.

Models and sizes come from ``XRL_MODEL`` / ``XRL_MODEL_NAME`` / ``XRL_MODEL_FLAVOR`` (student),
``XRL_TEACHER`` / ``XRL_TEACHER_NAME`` / ``XRL_TEACHER_FLAVOR``, ``XRL_NGPUS``, ``XRL_TOP_K`` ...
"""

from __future__ import annotations

import os

from meshy_b200.config import (InferenceServiceConfig, OPDTeacherConfig, OPDTrainingConfig, RolloutServiceConfig,
                               SamplingParams, TrainerConfig, TrainerParamsConfig)
from meshy_b200.service.base import ServiceGroup
from meshy_b200.service.colocation import ColocationRing, SchedulingMode
from meshy_b200.service.ignite import Ignitor

STUDENT_PATH = os.environ.get("XRL_MODEL") or None
STUDENT_NAME = os.environ.get("XRL_MODEL_NAME", "qwen3")
STUDENT_FLAVOR = os.environ.get("XRL_MODEL_FLAVOR", "1.7B")
TEACHER_PATH = os.environ.get("XRL_TEACHER") or None
TEACHER_NAME = os.environ.get("XRL_TEACHER_NAME", "qwen3")
TEACHER_FLAVOR = os.environ.get("XRL_TEACHER_FLAVOR", "8B")
NGPUS = int(os.environ.get("XRL_NGPUS", "1"))
TOPOLOGY = os.environ.get("XRL_TOPOLOGY", "colocate")
SEQ_LEN = int(os.environ.get("XRL_SEQ_LEN", "2048"))
MAX_NEW_TOKENS = int(os.environ.get("XRL_MAX_NEW_TOKENS", "1024"))
TOP_K = int(os.environ.get("XRL_TOP_K", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "4"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "4"))
BATCH_SIZE = ROLLOUT_BATCH * GROUP_SIZE
SCORE_BATCH = int(os.environ.get("XRL_SCORE_BATCH", str(BATCH_SIZE)))


def _tc(name: str, flavor: str, folder: str) -> TrainerConfig:
    return TrainerConfig(model_name=name, model_flavor=flavor, seq_len=SEQ_LEN, lr=float(os.environ.get("XRL_LR", "1e-6")),
                         steps=int(os.environ.get("XRL_STEPS", "1000")), weight_decay=0.0, dtype="bfloat16",
                         dp_shard_degree=-1, dp_replicate_degree=1, dump_folder=folder)


def _teacher() -> OPDTeacherConfig:
    return OPDTeacherConfig(model_path=TEACHER_PATH,
                            trainer_config=_tc(TEACHER_NAME, TEACHER_FLAVOR, "./outputs/student_topk_opd/teacher"),
                            top_k=TOP_K, score_batch_size=SCORE_BATCH)


def _student() -> OPDTrainingConfig:
    return OPDTrainingConfig(model_path=STUDENT_PATH,
                             trainer_config=_tc(STUDENT_NAME, STUDENT_FLAVOR, "./outputs/student_topk_opd/student"),
                             trainer_params=TrainerParamsConfig(mini_batch_size=1, batch_layout="packed",
                                                                max_tokens_per_micro=16384),
                             batch_size=BATCH_SIZE)


def _infer(n: int) -> InferenceServiceConfig:
    return InferenceServiceConfig(model_path=STUDENT_PATH,
                                  server_args={"model": f"{STUDENT_NAME}:{STUDENT_FLAVOR}", "context_length": SEQ_LEN})


def build_service_groups() -> list[ServiceGroup]:
    rollout = ServiceGroup(
        id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=["actor_train", "actor_infer", "teacher"],
        config=RolloutServiceConfig(model_path=STUDENT_PATH, dataset="meshy_b200.dataset.math:GSM8K",
                                    dataset_kwargs={"batch_size": ROLLOUT_BATCH, "seed": 42},
                                    reward="meshy_b200.dataset.math:GSM8K.reward",
                                    sampling_params=SamplingParams(max_new_tokens=MAX_NEW_TOKENS).as_dict(),
                                    group_size=GROUP_SIZE, pacing_window=1,
                                    num_epochs=int(os.environ.get("XRL_EPOCHS", "1"))))
    if TOPOLOGY == "colocate":
        return [ServiceGroup(id="actor_infer", n_replicas=NGPUS, n_gpus_per_replica=1, config=_infer(NGPUS)),
                ServiceGroup(id="teacher", n_replicas=1, n_gpus_per_replica=NGPUS, colocate_with="actor_infer",
                             wait_until=["actor_infer"], config=_teacher()),
                ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=NGPUS, colocate_with="actor_infer",
                             wait_until=["actor_infer", "teacher"], config=_student()),
                rollout]
    if TOPOLOGY == "disaggregate":
        n_teacher = int(os.environ.get("XRL_TEACHER_GPUS", "1"))
        rest = NGPUS - n_teacher
        if rest < 2:
            raise ValueError(f"disaggregate needs at least 2 cards besides the teacher's {n_teacher}")
        # the reference's split: XRL_TRAIN_GPUS trainer cards (default half, rounded down), the rest inference;
        # XRL_INFER_GPUS sets the inference side instead
        if "XRL_INFER_GPUS" in os.environ and "XRL_TRAIN_GPUS" not in os.environ:
            n_infer = int(os.environ["XRL_INFER_GPUS"])
            n_train = rest - n_infer
        else:
            n_train = int(os.environ.get("XRL_TRAIN_GPUS", str(max(1, rest // 2))))
            n_infer = rest - n_train
        if n_infer < 1 or n_train < 1:
            raise ValueError(f"disaggregate needs at least 1 inference and 1 trainer card (got {n_infer} / {n_train})")
        return [ServiceGroup(id="actor_infer", n_replicas=n_infer, n_gpus_per_replica=1, config=_infer(n_infer)),
                ServiceGroup(id="teacher", n_replicas=1, n_gpus_per_replica=n_teacher, wait_until=["actor_infer"],
                             config=_teacher()),
                ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=n_train,
                             wait_until=["actor_infer", "teacher"], config=_student()),
                rollout]
    raise ValueError(f"unknown XRL_TOPOLOGY={TOPOLOGY!r} (use 'colocate' or 'disaggregate')")


SERVICE_GROUPS = build_service_groups()
COLOCATIONS = ([ColocationRing(group_id="actor", ring=(("actor_infer", SchedulingMode.FALLBACK),
                                                       ("teacher", SchedulingMode.ON_DEMAND),
                                                       ("actor_train", SchedulingMode.ON_DEMAND)))]
               if TOPOLOGY == "colocate" else [])


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

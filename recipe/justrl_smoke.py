"""Smoke recipe: the JustRL service graph on a tiny Qwen3 (2 cards, CPU or GPU).

Same shape as ``recipe.justrl`` -- per-card inference replicas (``XRL_SMOKE_INFER_TP`` cards each:
tensor-parallel replicas) colocated with one DDP trainer in a FALLBACK / ON_DEMAND ring, plus the CPU
rollout driver --
on ``qwen3:debugmodel`` with synthetic token prompts and the parity reward,
for a few steps.  ``XRL_DEVICE=cpu`` runs it without a GPU (gloo):

    XRL_DEVICE=cpu python -m meshy_b200.launch --recipe recipe.justrl_smoke
"""

from __future__ import annotations

import os

from meshy_b200.config import (GlobalCheckpointConfig, InferenceServiceConfig, RolloutServiceConfig, SamplingParams,
                               TrainerConfig, TrainerParamsConfig, TrainingServiceConfig)
from meshy_b200.service.base import ServiceGroup
from meshy_b200.service.colocation import ColocationRing, SchedulingMode
from meshy_b200.service.ignite import Ignitor

MODEL = os.environ.get("XRL_SMOKE_MODEL", "qwen3:debugmodel")  # qwen3:debugmodel_moe for the MoE path
CARDS = int(os.environ.get("XRL_SMOKE_CARDS", "2"))
PROMPTS = int(os.environ.get("XRL_SMOKE_PROMPTS", "4"))
GROUP = 2
STEPS = int(os.environ.get("XRL_SMOKE_STEPS", "3"))
# "auto": CUDA IPC snapshots on a GPU node, the HF safetensors export on CPU
SYNC = os.environ.get("XRL_SMOKE_WEIGHT_SYNC", "auto")
CKPT = GlobalCheckpointConfig(enabled=os.environ.get("XRL_SMOKE_CKPT", "0") == "1", interval=1, keep_latest_k=2)


SHARD = os.environ.get("XRL_SMOKE_SHARD", "0") == "1"  # FSDP over the trainer's cards instead of DDP
INFER_TP = int(os.environ.get("XRL_SMOKE_INFER_TP", "1"))  # cards per inference replica (tensor parallel)
INFER_EP = int(os.environ.get("XRL_SMOKE_INFER_EP", "1"))  # = INFER_TP: the replica's ranks split the experts
_NAME, _FLAVOR = MODEL.split(":")
# pacing: "colocate" (default) shares every card; "disaggregate" puts inference on the first half of the cards
# and the trainer on the rest; XRL_SMOKE_PACING is the rollout's window ("none": no gate, fully async) and
# XRL_SMOKE_STREAM=1 lets the trainer take mini-batches as they arrive (disaggregated only)
TOPOLOGY = os.environ.get("XRL_SMOKE_TOPOLOGY", "colocate")
_pacing = os.environ.get("XRL_SMOKE_PACING", "1")
PACING = None if _pacing == "none" else int(_pacing)
STREAM = os.environ.get("XRL_SMOKE_STREAM", "0") == "1"
COLOCATE = TOPOLOGY == "colocate"
N_INFER = CARDS if COLOCATE else CARDS // 2
N_TRAIN = CARDS if COLOCATE else CARDS - N_INFER
if STREAM and COLOCATE:
    raise ValueError("XRL_SMOKE_STREAM=1 needs XRL_SMOKE_TOPOLOGY=disaggregate")


def _trainer_config() -> TrainerConfig:
    par = dict(shard_params="on", dp_shard_degree=-1, dp_replicate_degree=1) if SHARD else \
        dict(dp_replicate_degree=N_TRAIN)
    return TrainerConfig(model_name=_NAME, model_flavor=_FLAVOR, seq_len=512, lr=1e-5, weight_decay=0.0,
                         max_norm=1.0, steps=1000, dtype="bfloat16", **par)


SERVICE_GROUPS = [
    ServiceGroup(id="actor_infer", n_replicas=N_INFER // INFER_TP, n_gpus_per_replica=INFER_TP,
                 config=InferenceServiceConfig(model_path=None, server_args={
                     "model": MODEL, "max_running_requests": 16, "max_total_tokens": 8192, "context_length": 512,
                     **({"ep_size": INFER_EP} if INFER_EP > 1 else {})})),
    ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=N_TRAIN,
                 colocate_with="actor_infer" if COLOCATE else None, wait_until=["actor_infer"],
                 config=TrainingServiceConfig(
                     model_path=None, trainer_config=_trainer_config(),
                     trainer_params=TrainerParamsConfig(
                         mini_batch_size=GROUP if STREAM else PROMPTS * GROUP,
                         batch_layout="packed", max_tokens_per_micro=2048, old_logprobs_source="train"),
                     batch_size=PROMPTS * GROUP, weight_sync_mode=SYNC, checkpoint=CKPT, stream_minibatch=STREAM)),
    ServiceGroup(id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=["actor_train", "actor_infer"],
                 config=RolloutServiceConfig(
                     model_path=None, dataset="meshy_b200.dataset.synthetic:SyntheticPrompts",
                     dataset_kwargs={"batch_size": PROMPTS, "n_prompts": PROMPTS * STEPS, "vocab_size": 2048,
                                     "min_len": 8, "max_len": 24, "seed": 1},
                     reward="meshy_b200.dataset.synthetic:SyntheticPrompts.reward",
                     sampling_params=SamplingParams(max_new_tokens=24).as_dict(), group_size=GROUP,
                     poll_interval=0.2, pacing_window=PACING, num_epochs=1, checkpoint=CKPT,
                     async_max_running_request=-1 if PACING == 1 else 2 * PROMPTS * GROUP)),
]

COLOCATIONS = [ColocationRing(group_id="actor", ring=(("actor_infer", SchedulingMode.FALLBACK),
                                                      ("actor_train", SchedulingMode.ON_DEMAND)))] if COLOCATE else []


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

"""JustRL on Qwen3-30B-A3B (reference ``recipe/justrl_qwen3_30b_a3b.py``).

Trainer: 8 cards with expert parallelism EP8 (each rank owns 16 of the 128 experts; dense weights
data-parallel) -- new relative to the reference, whose trainer has no EP.  Inference: the reference needs
TP8 + EP8 because 60 GB of bf16 weights do not fit one 80 GB card; on a 180 GB B200 they do, so each card
runs a full single-card replica (replica-level data parallelism of inference instead of TP).
``XRL_INFER_TP=8`` gives the reference's layout instead: one tensor-parallel replica over the 8 cards, its
experts split over them by ``XRL_EP_SIZE`` (default: the replica's width; 1 keeps every expert on every
card). The reference's other variables apply too: ``XRL_MODEL`` (checkpoint dir), ``XRL_MEM_FRACTION`` (0.7),
``XRL_SEQ_LEN``, ``XRL_STEPS``, ``XRL_LR``, ``XRL_EPOCHS``."""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams, TrainerConfig, TrainerParamsConfig
from meshy_b200.recipe_lib import grpo_graph, model_from_env
from meshy_b200.service.ignite import Ignitor

NAME, FLAVOR, MODEL_PATH = model_from_env("qwen3", "30B-A3B")
NGPUS = int(os.environ.get("XRL_NGPUS", "8"))
ROLLOUT_BATCH = int(os.environ.get("XRL_ROLLOUT_BATCH", "32"))
GROUP_SIZE = int(os.environ.get("XRL_GROUP_SIZE", "8"))
SEQ_LEN = int(os.environ.get("XRL_SEQ_LEN", "16384"))
INFER_TP = int(os.environ.get("XRL_INFER_TP", "1"))
# the engine's KV cache takes this fraction of the memory left after the weights (SGLang's static fraction
# counts the weights too, hence a different default)
_server_args = {"mem_fraction_static": float(os.environ.get("XRL_MEM_FRACTION", "0.7"))}
if INFER_TP > 1:
    _server_args["ep_size"] = int(os.environ.get("XRL_EP_SIZE", str(INFER_TP)))

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=f"{NAME}:{FLAVOR}", model_path=MODEL_PATH,
    trainer_config=TrainerConfig(model_name=NAME, model_flavor=FLAVOR, seq_len=SEQ_LEN,
                                 steps=int(os.environ.get("XRL_STEPS", "3000")),
                                 lr=float(os.environ.get("XRL_LR", "1e-6")),
                                 weight_decay=0.1, dtype="bfloat16", dp_shard_degree=1, dp_replicate_degree=NGPUS,
                                 ep_degree=NGPUS, activation_checkpoint_mode="full",
                                 dump_folder="./outputs/justrl_qwen3_30b_a3b"),
    trainer_params=TrainerParamsConfig(mini_batch_size=1, batch_layout="packed", max_tokens_per_micro=16384,
                                       old_logprobs_source="train"),
    batch_size=ROLLOUT_BATCH * GROUP_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(max_new_tokens=int(os.environ.get("XRL_MAX_NEW_TOKENS", "15360"))), n_infer=NGPUS,
    server_args=_server_args, pacing_window=1, num_epochs=int(os.environ.get("XRL_EPOCHS", "1")),
    infer_tp=INFER_TP)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

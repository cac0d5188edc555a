"""JustRL fully asynchronous (reference ``recipe/justrl_fully_async.py``): disaggregated cards (4 inference,
4 training), no pacing gate (``pacing_window=None``), and the trainer streams mini-batches as they arrive
(``stream_minibatch``), syncing weights and the LR schedule once per full batch."""

from __future__ import annotations

import os

from meshy_b200.config import SamplingParams
from meshy_b200.recipe_lib import grpo_graph
from meshy_b200.service.ignite import Ignitor
from recipe.justrl import BATCH_SIZE, GROUP_SIZE, MODEL, MODEL_PATH, ROLLOUT_BATCH, trainer_config, trainer_params

N_INFER = int(os.environ.get("XRL_N_INFER", "4"))
N_TRAIN = int(os.environ.get("XRL_N_TRAIN", "4"))
_tc = trainer_config()
_tc.dp_replicate_degree = N_TRAIN

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=MODEL, model_path=MODEL_PATH, trainer_config=_tc, trainer_params=trainer_params(),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(max_new_tokens=15360), n_infer=N_INFER, n_train=N_TRAIN, colocate=False,
    pacing_window=None, async_max_running_request=int(BATCH_SIZE * 1.5), stream_minibatch=True, num_epochs=8)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

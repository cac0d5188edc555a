"""JustRL with bounded off-policy pacing (reference ``recipe/justrl_async.py``): the rollout may run one
window ahead of the trainer (``pacing_window=2``) with up to 1.5 x batch samples in flight."""

from __future__ import annotations

from meshy_b200.config import SamplingParams
from meshy_b200.recipe_lib import grpo_graph
from meshy_b200.service.ignite import Ignitor
from recipe.justrl import BATCH_SIZE, GROUP_SIZE, MODEL, MODEL_PATH, NGPUS, ROLLOUT_BATCH, trainer_config, trainer_params

SERVICE_GROUPS, COLOCATIONS = grpo_graph(
    model=MODEL, model_path=MODEL_PATH, trainer_config=trainer_config(), trainer_params=trainer_params(),
    batch_size=BATCH_SIZE, rollout_batch=ROLLOUT_BATCH, group_size=GROUP_SIZE,
    dataset="meshy_b200.dataset.math:MATH", dataset_kwargs={"seed": 42}, reward="meshy_b200.dataset.math:MATH.reward",
    sampling=SamplingParams(max_new_tokens=15360), n_infer=NGPUS, pacing_window=2,
    async_max_running_request=int(BATCH_SIZE * 1.5), num_epochs=8)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

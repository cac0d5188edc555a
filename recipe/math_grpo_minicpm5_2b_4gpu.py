"""Long-context math GRPO on MiniCPM5-2B, 4 cards (reference ``recipe/math_grpo_minicpm5_2b_4gpu.py``)."""

from __future__ import annotations

from meshy_b200.service.ignite import Ignitor
from recipe.math_grpo_minicpm5_2b import build

SERVICE_GROUPS, COLOCATIONS = build(ngpus=4, rollout_batch=128, batch_size=256)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

"""JustRL on MiniCPM5-2B over 4 cards (reference ``recipe/justrl_minicpm5_2b_4gpu.py``)."""

from __future__ import annotations

from meshy_b200.service.ignite import Ignitor
from recipe.justrl_minicpm5_2b import build

SERVICE_GROUPS, COLOCATIONS = build("2B", ngpus=4)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

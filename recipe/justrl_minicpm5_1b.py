"""JustRL on MiniCPM5-1B (reference ``recipe/justrl_minicpm5_1b.py``): the 2B recipe with the 1B flavour."""

from __future__ import annotations

from meshy_b200.service.ignite import Ignitor
from recipe.justrl_minicpm5_2b import build

SERVICE_GROUPS, COLOCATIONS = build("1B")


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

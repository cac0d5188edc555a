"""The 128k JustRL-II recipe on 32 cards (reference ``recipe/justrl_ii_minicpm5_2b_128k_32gpu.py``).

16 cards: inference replicas time-sharing with the CP4 x DP4 actor; 16 dedicated cards: the CP4 x DP4
critic (30 cold-start windows by default).  Launch one launcher per node with the same recipe
(``python -m meshy_b200.launch --recipe recipe.justrl_ii_minicpm5_2b_128k_32gpu --nnodes 4
--nproc-per-node 8 --node-rank R --master-addr HOST``).
"""

from __future__ import annotations

import os

from meshy_b200.service.ignite import Ignitor
from recipe.justrl_ii_minicpm5_2b_128k import build

os.environ.setdefault("XRL_COLD_START_WINDOWS", "30")
SERVICE_GROUPS, COLOCATIONS = build(ngpus=16, critic_colocate=False, n_critic=16)


def main() -> None:
    Ignitor(SERVICE_GROUPS, COLOCATIONS).run()


if __name__ == "__main__":
    main()

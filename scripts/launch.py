"""Run launcher at the reference's path: ``python scripts/launch.py --recipe recipe.justrl``.

The launcher itself is :mod:`meshy_b200.launch` (``python -m meshy_b200.launch`` is the same command), with
the reference launcher's flags: ``--recipe``, ``--nnodes``, ``--node-rank``, ``--master-addr``,
``--master-port``, ``--nproc-per-node``, ``--runtime-dir``, ``--resume``, ``--checkpoint-dir``, ``--log-dir``,
``--tensorboard-dir``, ``--trajectory-dir``. The reference's analysis and benchmark scripts are the modules
``meshy_b200.bench.analyze`` (``step-timing`` / ``rewards``) and ``meshy_b200.bench.train_only``.
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from meshy_b200.launch import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())

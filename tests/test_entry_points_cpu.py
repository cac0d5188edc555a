"""``python scripts/launch.py`` (the reference's launcher path) is the package launcher with the reference
launcher's flags."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_scripts_launch_has_the_reference_flags():
    r = subprocess.run([sys.executable, "scripts/launch.py", "--help"], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    for flag in ("--recipe", "--nnodes", "--node-rank", "--master-addr", "--master-port", "--nproc-per-node",
                 "--runtime-dir", "--resume", "--checkpoint-dir", "--log-dir", "--tensorboard-dir",
                 "--trajectory-dir"):
        assert flag in r.stdout, flag

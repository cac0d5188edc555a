"""Import hygiene (CPU): the GRPO mainline loads neither the on-policy-distillation nor the critic stack, and
nothing in the package pulls in a compatibility layer or another library's attention / GEMM kernels (Triton,
flash-attn, FlashInfer, vLLM). Checked in a fresh interpreter so earlier tests cannot have loaded them."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MAINLINE = ["meshy_b200", "meshy_b200.rl", "meshy_b200.backend.trainer", "meshy_b200.rollout.engine",
            "meshy_b200.service.training", "meshy_b200.service.rollout", "meshy_b200.worker.rollout",
            "meshy_b200.ops.functional", "meshy_b200.ops.decode", "meshy_b200.parallel.symm", "recipe.justrl"]
OPD = ["meshy_b200.backend.opd", "meshy_b200.backend.topk_loss", "meshy_b200.engine.opd", "meshy_b200.worker.opd",
       "meshy_b200.service.opd"]
CRITIC = ["meshy_b200.backend.critic", "meshy_b200.engine.critic", "meshy_b200.worker.critic",
          "meshy_b200.service.critic"]
FOREIGN = ["triton", "flash_attn", "flashinfer", "vllm", "sglang", "tilelang"]


def test_mainline_imports_stay_clean():
    code = (
        "import importlib, json, sys\n"
        f"for m in {MAINLINE!r}: importlib.import_module(m)\n"
        "print(json.dumps(sorted(sys.modules)))\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    loaded = set(json.loads(r.stdout.strip().splitlines()[-1]))
    assert not [m for m in OPD if m in loaded], "OPD modules loaded by the GRPO mainline"
    assert not [m for m in CRITIC if m in loaded], "critic modules loaded by the GRPO mainline"
    foreign = [m for m in loaded if m.split(".")[0] in FOREIGN]
    assert not foreign, f"foreign kernel libraries imported: {sorted(foreign)[:10]}"

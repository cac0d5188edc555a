"""Recipes honour the reference recipes' environment variables (each case imports the recipe in a fresh
interpreter, since recipes read the environment at import): model selection (``XRL_MODEL`` as a checkpoint
path or a registry spec, ``XRL_MODEL_NAME`` / ``XRL_MODEL_FLAVOR``), ``XRL_STEPS`` / ``XRL_LR``,
``XRL_TOPOLOGY`` + ``XRL_TRAIN_GPUS`` card splits, ``XRL_EP_SIZE`` / ``XRL_MEM_FRACTION`` with tensor-parallel
inference replicas, and the ``XRL_CHECKPOINT*`` switches."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROBE = r"""
import importlib, json, sys
m = importlib.import_module(sys.argv[1])
out = {"groups": {g.id: [g.n_replicas, g.n_gpus_per_replica, g.colocate_with] for g in m.SERVICE_GROUPS}}
for g in m.SERVICE_GROUPS:
    c = g.config
    tc = getattr(c, "trainer_config", None)
    if tc is not None:
        out.setdefault("trainer", {})[g.id] = [tc.model_name, tc.model_flavor, tc.steps, tc.lr]
    if hasattr(c, "server_args"):
        out["server_args"] = c.server_args
        out["infer_path"] = c.model_path
    ck = getattr(c, "checkpoint", None)
    if ck is not None:
        out.setdefault("checkpoint", {})[g.id] = [ck.enabled, ck.interval, ck.keep_latest_k]
print(json.dumps(out))
"""


def _probe(module, **env):
    e = {k: v for k, v in os.environ.items() if not k.startswith("XRL_") and k != "MODEL_PATH"}
    e.update(env, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", _PROBE, module], env=e, cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_grpo_gsm8k_variables(tmp_path):
    d = _probe("recipe.grpo_gsm8k")
    assert d["groups"]["actor_infer"] == [1, 1, None] and d["groups"]["actor_train"] == [1, 1, "actor_infer"]
    assert d["trainer"]["actor_train"] == ["qwen3", "1.7B", 1000, 1e-6]
    assert d["infer_path"] is None  # the hub id has no local copy: random-init weights
    d = _probe("recipe.grpo_gsm8k", XRL_NGPUS="4", XRL_TOPOLOGY="disaggregate", XRL_TRAIN_GPUS="1",
               XRL_STEPS="77", XRL_LR="3e-6", XRL_MODEL="qwen3:0.6B")
    assert d["groups"]["actor_infer"] == [3, 1, None] and d["groups"]["actor_train"] == [1, 1, None]
    assert d["trainer"]["actor_train"] == ["qwen3", "0.6B", 77, 3e-6]
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    d = _probe("recipe.grpo_gsm8k", XRL_MODEL=str(ckpt), XRL_MODEL_NAME="qwen2_5", XRL_MODEL_FLAVOR="1.5B",
               XRL_NGPUS="8", XRL_INFER_TP="2")
    assert d["infer_path"] == str(ckpt) and d["trainer"]["actor_train"][:2] == ["qwen2_5", "1.5B"]
    assert d["groups"]["actor_infer"] == [4, 2, None] and d["groups"]["actor_train"] == [1, 8, "actor_infer"]


def test_moe_recipe_expert_parallel_inference():
    d = _probe("recipe.justrl_qwen3_30b_a3b")
    assert d["groups"]["actor_infer"] == [8, 1, None] and "ep_size" not in d["server_args"]
    d = _probe("recipe.justrl_qwen3_30b_a3b", XRL_INFER_TP="8", XRL_MEM_FRACTION="0.5", XRL_STEPS="5")
    assert d["groups"]["actor_infer"] == [1, 8, None]
    assert d["server_args"]["ep_size"] == 8 and d["server_args"]["tp_size"] == 8
    assert d["server_args"]["mem_fraction_static"] == 0.5 and d["trainer"]["actor_train"][2] == 5
    d = _probe("recipe.justrl_qwen3_30b_a3b", XRL_INFER_TP="8", XRL_EP_SIZE="1")
    assert d["server_args"]["ep_size"] == 1


def test_opd_card_split_and_checkpoint_switches():
    d = _probe("recipe.student_topk_opd", XRL_NGPUS="8", XRL_TOPOLOGY="disaggregate", XRL_TEACHER_GPUS="1")
    # the reference's split of the 7 non-teacher cards: 3 trainer cards (half, rounded down), 4 inference
    assert d["groups"]["actor_train"][1] == 3 and d["groups"]["actor_infer"][0] == 4
    d = _probe("recipe.student_topk_opd", XRL_NGPUS="8", XRL_TOPOLOGY="disaggregate", XRL_TRAIN_GPUS="5")
    assert d["groups"]["actor_train"][1] == 5 and d["groups"]["actor_infer"][0] == 2
    d = _probe("recipe.justrl_ii_minicpm5_2b")
    assert d["checkpoint"]["actor_train"] == [True, 10, 3]
    d = _probe("recipe.justrl_ii_minicpm5_2b", XRL_CHECKPOINT="0", XRL_CHECKPOINT_KEEP="5")
    assert d["checkpoint"]["actor_train"][0] is False and d["checkpoint"]["actor_train"][2] == 5

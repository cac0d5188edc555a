"""Every shipped recipe imports, builds its service graph and places it on the cards it asks for.

Mirrors the reference's recipe-level checks (``tests/test_recipe_*.py``): the graph must be valid for
``build_topology`` (colocation rings, card blocks, wait-until edges), and a few recipe-specific facts
hold (parallel degrees, trainer field lists, placement of dedicated critics).
"""

import importlib
import pkgutil

import pytest

import recipe
from meshy_b200.config import GAE_TRAINER_FIELDS
from meshy_b200.service.base import GPU
from meshy_b200.service.topology import build_topology

RECIPES = sorted(m.name for m in pkgutil.iter_modules(recipe.__path__))


def _cards(groups) -> int:
    return sum(g.n_replicas * g.n_gpus_per_replica for g in groups if not g.colocate_with)


@pytest.mark.parametrize("name", RECIPES)
def test_recipe_builds_topology(name):
    mod = importlib.import_module(f"recipe.{name}")
    groups, rings = mod.SERVICE_GROUPS, mod.COLOCATIONS
    assert callable(mod.main)
    n = _cards(groups)
    per_node = min(n, 8) or 1
    gpus = [GPU(global_rank=i, host=f"node{i // per_node}", local_rank=i % per_node, node_rank=i // per_node)
            for i in range(max(n, 1))]
    topo = build_topology(groups, gpus, rings)
    ids = {s.group_id for s in topo.services}
    assert {g.id for g in groups} == ids
    assert "rollout" in ids


def test_recipe_specifics():
    r = importlib.import_module("recipe.justrl_ii_minicpm5_2b")
    critic = next(g for g in r.SERVICE_GROUPS if g.id == "critic")
    train = next(g for g in r.SERVICE_GROUPS if g.id == "actor_train")
    assert critic.colocate_with is None and critic.n_gpus_per_replica == 4
    assert train.config.tq_fields == list(GAE_TRAINER_FIELDS)
    r = importlib.import_module("recipe.justrl_ii_minicpm5_2b_128k")
    train = next(g for g in r.SERVICE_GROUPS if g.id == "actor_train")
    assert train.config.trainer_config.cp_degree == 4 and train.config.trainer_config.dp_replicate_degree == 2
    assert "positive_lm_weight" in train.config.tq_fields
    r = importlib.import_module("recipe.justrl_ii_resume_smoke")
    train = next(g for g in r.SERVICE_GROUPS if g.id == "actor_train")
    assert "advantage" in train.config.tq_fields  # the critic publishes finished advantages
    r = importlib.import_module("recipe.justrl_qwen3_30b_a3b")
    train = next(g for g in r.SERVICE_GROUPS if g.id == "actor_train")
    assert train.config.trainer_config.ep_degree == 8
    r = importlib.import_module("recipe.justrl_minicpm5_1b")
    train = next(g for g in r.SERVICE_GROUPS if g.id == "actor_train")
    assert train.config.trainer_config.model_flavor == "1B"

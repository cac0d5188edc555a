"""Building blocks for recipes: the standard service graphs as one function call.

A recipe is a module exporting ``SERVICE_GROUPS``, ``COLOCATIONS`` and
``main()`` (reference ``recipe/justrl.py:154-167``).  Most recipes are one of
three graphs, which :func:`grpo_graph` builds:

* **colocated** (``colocate=True``): ``n_infer`` single-card inference replicas (or ``n_infer / infer_tp``
  tensor-parallel ones)
  and one trainer replica on the same cards, handing them over through a
  FALLBACK (inference) / ON_DEMAND (trainer [, critic]) ring;
* **disaggregated** (``colocate=False``): inference on the first ``n_infer``
  cards, the trainer on the next ``n_train``;
* optionally a critic replica sharing the trainer's cards and ring
  (PPO with VAPO-GAE; the rollout then leaves the advantage to the critic).

The rollout driver (CPU) is always added last with ``wait_until`` on the GPU
groups.  Knobs keep the reference's names (``pacing_window``,
``async_max_running_request``, ``stream_minibatch`` ...).
"""

from __future__ import annotations

from typing import Any

from .config import (GAE_TRAINER_FIELDS, GRPO_TRAINER_FIELDS, CriticServiceConfig, GlobalCheckpointConfig, InferenceServiceConfig,
                     RolloutServiceConfig, SamplingParams, TrainerConfig, TrainerParamsConfig,
                     TrainingServiceConfig)
from .service.base import ServiceGroup
from .service.colocation import ColocationRing, SchedulingMode


def grpo_graph(*, model: str, model_path: str | None, trainer_config: TrainerConfig,
               trainer_params: TrainerParamsConfig, batch_size: int, rollout_batch: int, group_size: int,
               dataset: str, dataset_kwargs: dict | None = None, reward: str | None = None,
               sampling: SamplingParams | None = None, n_infer: int = 8, n_train: int | None = None,
               colocate: bool = True, pacing_window: int | str | None = 1, async_max_running_request: int = -1,
               stream_minibatch: bool = False, server_args: dict | None = None,
               critic: CriticServiceConfig | None = None, checkpoint: GlobalCheckpointConfig | None = None,
               advantage: str | None = None, reward_shaping: str | None = None,
               reward_shaping_kwargs: dict | None = None, filter_zero_std_groups: bool = False,
               oversample_factor: float = 1.0, num_epochs: int = 1,
               trainer_service: type = TrainingServiceConfig, trainer_extra: dict | None = None,
               extra_groups: list[ServiceGroup] | None = None, ring_extra: list[tuple[str, Any]] | None = None,
               critic_colocate: bool | None = None, n_critic: int | None = None, rollout_extra: dict | None = None,
               infer_tp: int = 1):
    """Service groups and colocation rings of one GRPO / PPO run (see the module docstring).

    ``critic_colocate=False`` gives the critic its own ``n_critic`` cards (declared after the
    inference cards, so they follow them); ``rollout_extra`` passes further
    :class:`RolloutServiceConfig` fields (``advantage_kwargs``, ``verbose_trajectory_log`` ...).
    ``infer_tp`` > 1 makes each inference replica a tensor-parallel group of that many cards (the ``n_infer``
    cards then hold ``n_infer / infer_tp`` replicas).
    """
    if stream_minibatch and colocate:
        raise ValueError("stream_minibatch needs disaggregated cards (it is incompatible with colocation)")
    n_train = n_infer if n_train is None else n_train
    ckpt = checkpoint or GlobalCheckpointConfig()
    sargs = {"model": model, "tp_size": 1}
    sargs.update(server_args or {})
    if infer_tp < 1 or n_infer % infer_tp:
        raise ValueError(f"{n_infer} inference cards do not split into replicas of {infer_tp}")
    sargs["tp_size"] = infer_tp
    infer = ServiceGroup(id="actor_infer", n_replicas=n_infer // infer_tp, n_gpus_per_replica=infer_tp,
                         config=InferenceServiceConfig(model_path=model_path, server_args=sargs))
    groups = [infer]
    ring = [("actor_infer", SchedulingMode.FALLBACK)]
    waits_train = ["actor_infer"]
    if critic is not None:
        c_colo = colocate if critic_colocate is None else critic_colocate
        groups.append(ServiceGroup(id="critic", n_replicas=1, n_gpus_per_replica=n_critic or n_train,
                                   colocate_with="actor_infer" if c_colo else None,
                                   wait_until=["actor_infer"], config=critic))
        if c_colo:
            ring.append(("critic", SchedulingMode.ON_DEMAND))
        waits_train.append("critic")
    tkw = dict(model_path=model_path, trainer_config=trainer_config, trainer_params=trainer_params,
               batch_size=batch_size, stream_minibatch=stream_minibatch, checkpoint=ckpt)
    fields = list(GRPO_TRAINER_FIELDS)
    if critic is not None:
        if critic.publish_mode == "values":  # the trainer computes GAE from the critic's values
            fields = list(GAE_TRAINER_FIELDS)
        tkw["critic_cold_start_windows"] = critic.cold_start_windows
    if (rollout_extra or {}).get("publish_positive_lm_weights"):
        fields.append("positive_lm_weight")
    if fields != GRPO_TRAINER_FIELDS:
        tkw["tq_fields"] = fields
    tkw.update(trainer_extra or {})
    groups.append(ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=n_train,
                               colocate_with="actor_infer" if colocate else None, wait_until=waits_train,
                               config=trainer_service(**tkw)))
    ring.append(("actor_train", SchedulingMode.ON_DEMAND))
    groups += list(extra_groups or [])
    ring += list(ring_extra or [])
    groups.append(ServiceGroup(
        id="rollout", n_replicas=1, n_gpus_per_replica=0, wait_until=[g.id for g in groups if g.uses_gpu],
        config=RolloutServiceConfig(
            model_path=model_path, dataset=dataset, dataset_kwargs=dict(dataset_kwargs or {}, batch_size=rollout_batch),
            reward=reward, reward_shaping=reward_shaping, reward_shaping_kwargs=dict(reward_shaping_kwargs or {}),
            advantage=advantage, sampling_params=(sampling or SamplingParams()).as_dict(), group_size=group_size,
            pacing_window=pacing_window, async_max_running_request=async_max_running_request, num_epochs=num_epochs,
            filter_zero_std_groups=filter_zero_std_groups, oversample_factor=oversample_factor,
            external_advantage=critic is not None, checkpoint=ckpt, **(rollout_extra or {}))))
    colocations = [ColocationRing(group_id="actor", ring=tuple(ring))] if colocate else []
    return groups, colocations


__all__ = ["grpo_graph"]


def model_from_env(name: str, flavor: str, *, path_env: str = "XRL_MODEL") -> tuple[str, str, str | None]:
    """``(registry name, flavor, checkpoint dir or None)`` of a recipe's model, with the reference recipes'
    variables: ``XRL_MODEL`` names the checkpoint (a local directory; a hub id without a local copy gives
    random-init weights of the architecture, there being no network), ``XRL_MODEL_NAME`` / ``XRL_MODEL_FLAVOR``
    the architecture. ``XRL_MODEL=name:flavor`` (a registry spec, no such directory) also selects the
    architecture; ``MODEL_PATH`` is accepted as the checkpoint too."""
    import os

    spec = os.environ.get(path_env, "")
    path = os.environ.get("MODEL_PATH") or None
    if spec and ":" in spec and "/" not in spec and not os.path.isdir(spec):
        name, flavor = spec.split(":", 1)
    elif spec:
        path = spec
    name = os.environ.get("XRL_MODEL_NAME", name)
    flavor = os.environ.get("XRL_MODEL_FLAVOR", flavor)
    path = os.path.abspath(os.path.expanduser(path)) if path and os.path.isdir(os.path.expanduser(path)) else None
    return name, flavor, path


def checkpoint_from_env(interval: int = 10, keep_latest_k: int = 2, enabled: bool = True) -> GlobalCheckpointConfig:
    """Global checkpoint policy with the reference recipes' switches: ``XRL_CHECKPOINT`` (``0`` / ``false`` /
    empty turn it off), ``XRL_CHECKPOINT_INTERVAL``, ``XRL_CHECKPOINT_KEEP``."""
    import os

    on = os.environ.get("XRL_CHECKPOINT", "1" if enabled else "0").strip().lower() not in ("0", "false", "")
    return GlobalCheckpointConfig(enabled=on, interval=int(os.environ.get("XRL_CHECKPOINT_INTERVAL", interval)),
                                  keep_latest_k=int(os.environ.get("XRL_CHECKPOINT_KEEP", keep_latest_k)))


def local_model_path(env: str = "MINICPM5_LOCAL_PATH", default: str | None = None) -> str | None:
    """Checkpoint directory from ``env`` (``None``: random-init weights of the named architecture)."""
    import os

    p = os.environ.get(env) or default
    return os.path.abspath(os.path.expanduser(p)) if p else None


__all__ += ["checkpoint_from_env", "local_model_path", "model_from_env"]

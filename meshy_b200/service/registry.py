"""Lazy ``"module:Class"`` resolution of role plugins (reference ``meshy/service/registry.py``)."""

from __future__ import annotations

import importlib
from typing import Any

SERVICE_TYPES = {
    "inference": "meshy_b200.service.inference:InferenceService",
    "training": "meshy_b200.service.training:TrainingService",
    "rollout": "meshy_b200.service.rollout:RolloutService",
    "critic": "meshy_b200.service.critic:CriticService",
    "teacher": "meshy_b200.service.opd:OPDTeacherService",
}


def resolve_callable(spec: str | Any) -> Any:
    if not isinstance(spec, str):
        return spec
    if ":" not in spec:
        raise ValueError(f"expected 'module:attr', got {spec!r}")
    mod, attr = spec.split(":", 1)
    obj = importlib.import_module(mod)
    for part in attr.split("."):
        obj = getattr(obj, part)
    return obj


def resolve_service(config) -> type:
    spec = getattr(type(config), "service_cls", "") or SERVICE_TYPES.get(type(config).role, "")
    if not spec:
        raise ValueError(f"{type(config).__name__} declares no service_cls and role {type(config).role!r} is unknown")
    return resolve_callable(spec)


__all__ = ["SERVICE_TYPES", "resolve_callable", "resolve_service"]

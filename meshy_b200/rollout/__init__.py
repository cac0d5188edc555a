"""Rollout engine: paged KV, continuous batching, CUDA-graph decode, HTTP API."""

from .engine import Generation, Request, RolloutEngine

__all__ = ["Generation", "Request", "RolloutEngine"]

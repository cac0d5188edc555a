"""PPO critic: value model, window batching, value training and health gauges."""

from .model import CriticModel, critic_args_from_actor

__all__ = ["CriticModel", "critic_args_from_actor"]

"""meshy_b200: a Blackwell-native asynchronous RL engine for LLMs.

Layers (top to bottom): recipes and launcher, services (topology, ignitor,
colocation ring, checkpoints), workers (TransferQueue-driven role loops),
engines (trainer, critic, teacher, rollout client), the training backend
(PPO/GRPO, planner, batch layout, critic/GAE, OPD), the native data plane,
the rollout engine, and the sm_100a kernel library.
"""

__version__ = "0.1.0"

"""Typed configuration contract of the framework.

Every recipe builds its run out of these dataclasses; they are the plugin
contract between recipes, services, workers and engines.  The class names and
field names follow the reference's schema (``meshy/config.py:14-588``) so a
recipe written against the reference reads the same here.  What differs is the
engine behind them: ``service_cls`` strings point at this package's services
(native rollout engine instead of SGLang, native trainer instead of
torchtitan), and the trainer config grows the knobs of the B200 trainer
(``ep_degree``, ``weight_sync_mode="device"``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, ClassVar, Literal


@dataclass
class SamplingParams:
    """Decode sampling knobs (reference ``meshy/config.py:14-27``)."""

    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_new_tokens: int = 16384

    def as_dict(self) -> dict[str, Any]:
        return {
            "temperature": self.temperature,
            "top_p": self.top_p,
            "top_k": self.top_k,
            "max_new_tokens": self.max_new_tokens,
        }


@dataclass(frozen=True)
class GlobalCheckpointConfig:
    """Shared checkpoint clock and retention for every checkpointing service.

    Each role writes its own shard at global window ``step`` when
    ``step % interval == 0``; the resume point is the newest step every
    participant committed (reference ``meshy/config.py:30-80``).  Retaining a
    single step could leave the intersection empty while a slower peer is
    still writing the newest one, hence ``keep_latest_k >= 2``.
    """

    enabled: bool = False
    interval: int = 10
    keep_latest_k: int = 3

    def __post_init__(self) -> None:
        if self.interval <= 0:
            raise ValueError(f"checkpoint interval must be positive, got {self.interval!r}")
        if self.keep_latest_k < 2:
            raise ValueError(
                "checkpoint keep_latest_k must be >= 2 so the resume intersection "
                f"can never be empty (got {self.keep_latest_k!r})"
            )

    def due(self, global_step: int) -> bool:
        return self.enabled and global_step > 0 and global_step % self.interval == 0

    @classmethod
    def coerce(cls, value: "GlobalCheckpointConfig | dict | None") -> "GlobalCheckpointConfig":
        if value is None:
            return cls()
        if isinstance(value, cls):
            return value
        return cls(**value)


@dataclass
class TrainerConfig:
    """Model + optimiser + parallelism of one training replica.

    Reference ``meshy/config.py:83-146``.  ``ep_degree`` is new: the reference
    trains MoE models as plain FSDP, this trainer can shard experts.
    """

    model_name: str = "qwen3"
    model_flavor: str = "1.7B"
    seq_len: int = 2048
    steps: int = 100
    dtype: str = "bfloat16"
    max_norm: float = 1.0
    local_batch_size: int = 4
    global_batch_size: int = -1
    lr: float = 1e-5
    weight_decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    warmup_steps: int = 0
    lr_decay_ratio: float | None = 0.0
    lr_decay_type: Literal["linear", "sqrt", "cosine"] = "linear"
    lr_min_factor: float = 0.0
    dp_shard_degree: int = -1
    dp_replicate_degree: int = 1
    # parameter sharding over the dp_shard ranks: "on" always (FSDP; HSDP with dp_replicate_degree > 1),
    # "off" never (parameters replicated, AdamW state and fp32 master sharded inside the fused DP step),
    # "auto" when the replicated training state would take more than 40 % of a device's memory
    shard_params: Literal["auto", "on", "off"] = "auto"
    tp_degree: int = 1
    cp_degree: int = 1
    ep_degree: int = 1
    enable_checkpoint: bool = False
    checkpoint_folder: str = "checkpoint"
    dump_folder: str = "./outputs"
    # Accepted for recipe compatibility; this trainer never uses a tracing
    # compiler (hot ops are hand-written kernels, inner loops CUDA graphs).
    compile_model: bool = False
    compile_backend: str = "none"
    activation_checkpoint_mode: Literal["selective", "full", "memory_budget", "none"] = "selective"
    attn_backend: Literal["sdpa", "varlen"] = "sdpa"

    def __post_init__(self) -> None:
        if self.attn_backend not in ("sdpa", "varlen"):
            raise ValueError(f"attn_backend must be 'sdpa' or 'varlen', got {self.attn_backend!r}")
        if self.lr_decay_ratio is not None and not (0.0 <= self.lr_decay_ratio <= 1.0):
            raise ValueError(f"lr_decay_ratio must be None or within [0, 1], got {self.lr_decay_ratio!r}")
        if self.lr_decay_type not in ("linear", "sqrt", "cosine"):
            raise ValueError(f"lr_decay_type must be 'linear', 'sqrt' or 'cosine', got {self.lr_decay_type!r}")
        if not (0.0 <= self.lr_min_factor <= 1.0):
            raise ValueError(f"lr_min_factor must be within [0, 1], got {self.lr_min_factor!r}")
        if self.shard_params not in ("auto", "on", "off"):
            raise ValueError(f"shard_params must be 'auto', 'on' or 'off', got {self.shard_params!r}")
        for name in ("tp_degree", "cp_degree", "ep_degree", "dp_replicate_degree"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")


@dataclass
class TrainerParamsConfig:
    """PPO / batching hyper-parameters (reference ``meshy/config.py:149-232``)."""

    mini_batch_size: int = 1
    micro_batch_size: int = 1
    batch_layout: Literal["padded", "packed"] = "padded"
    max_tokens_per_micro: int | None = None
    seq_bucket: int = 2048
    ppo_clip_eps_low: float = 0.2
    ppo_clip_eps_high: float = 0.2
    old_logprobs_source: Literal["rollout", "train"] = "rollout"
    calculate_per_token_loss: bool = False
    use_tis: bool = False
    use_icepop: bool = False
    positive_lm_loss_coef: float = 0.0
    tis_ratio_min: float = 0.5
    tis_ratio_max: float = 5.0
    logprob_chunk_size: int = 1024
    log_entropy: bool = True
    entropy_chunk_size: int = 512
    enable_gae: bool = False
    normalize_advantages: bool = False
    gae_gamma: float = 1.0
    gae_alpha: float = 1.5
    gae_lambda: float | None = None

    def __post_init__(self) -> None:
        if self.entropy_chunk_size <= 0:
            raise ValueError("entropy_chunk_size must be positive")
        if self.use_icepop and self.old_logprobs_source != "train":
            raise ValueError("IcePop requires old_logprobs_source='train'")
        if self.positive_lm_loss_coef < 0:
            raise ValueError("positive_lm_loss_coef must be nonnegative")
        if self.normalize_advantages and not self.enable_gae:
            raise ValueError("normalize_advantages requires enable_gae")
        if self.positive_lm_loss_coef and self.enable_gae and self.gae_gamma != 1.0:
            raise ValueError("Positive LM reward gating requires undiscounted returns (gae_gamma=1)")
        if not 0.0 <= self.gae_gamma <= 1.0:
            raise ValueError(f"gae_gamma must be within [0, 1], got {self.gae_gamma!r}")
        if self.gae_alpha <= 0:
            raise ValueError("gae_alpha must be positive")
        if self.gae_lambda is not None and not 0.0 <= self.gae_lambda <= 1.0:
            raise ValueError(f"gae_lambda must be None or within [0, 1], got {self.gae_lambda!r}")
        if self.old_logprobs_source not in ("rollout", "train"):
            raise ValueError(f"old_logprobs_source must be 'rollout' or 'train', got {self.old_logprobs_source!r}")
        if self.tis_ratio_min <= 0 or self.tis_ratio_max < self.tis_ratio_min:
            raise ValueError("TIS ratio bounds must satisfy 0 < min <= max")
        if self.logprob_chunk_size <= 0:
            raise ValueError("logprob_chunk_size must be positive")
        if self.batch_layout not in ("padded", "packed"):
            raise ValueError(f"batch_layout must be 'padded' or 'packed', got {self.batch_layout!r}")
        if self.max_tokens_per_micro is not None and self.max_tokens_per_micro <= 0:
            raise ValueError("max_tokens_per_micro must be positive when set")
        if self.batch_layout == "packed" and self.max_tokens_per_micro is None:
            raise ValueError("batch_layout='packed' requires max_tokens_per_micro")
        if self.seq_bucket <= 0:
            raise ValueError("seq_bucket must be positive")


@dataclass
class ServiceConfig:
    """Base of every role config: the role's plugin identity and port bases."""

    role: ClassVar[str] = "?"
    service_cls: ClassVar[str] = ""
    uses_gpu: ClassVar[bool] = True
    endpoint_port_base: ClassVar[int | None] = None
    dist_port_base: ClassVar[int | None] = None


DEFAULT_DATA_PARTITION = "data.train"

#: Columns the rollout writes per sample and the trainer fetches; the
#: trainer's fetch is an AND-filter over them (reference ``meshy/config.py:248-261``).
GRPO_TRAINER_FIELDS = [
    "tokens",
    "logprobs",
    "mask_assistant",
    "advantage",
    "weight_version",
    "reward",
    "truncated",
    "repetition",
    "mixed_version",
]


@dataclass
class InferenceServiceConfig(ServiceConfig):
    """A rollout-engine replica (the native paged-KV engine, HTTP front end).

    ``server_args`` keeps the SGLang-style keys recipes already use
    (``tp_size``, ``ep_size``, ``mem_fraction_static``, ``enable_memory_saver``,
    ``max_running_requests``, ``max_total_tokens`` ...).
    """

    role: ClassVar[str] = "inference"
    service_cls: ClassVar[str] = "meshy_b200.service.inference:InferenceService"
    endpoint_port_base: ClassVar[int] = 30000
    dist_port_base: ClassVar[int] = 40000

    model_path: str | None = None
    server_args: dict[str, Any] = field(default_factory=dict)


@dataclass
class TrainingServiceConfig(ServiceConfig):
    """The actor trainer replica (reference ``meshy/config.py:275-312``).

    ``weight_sync_mode``: ``"device"`` pushes weights straight into the
    colocated/disaggregated engines' weight buffers over CUDA IPC / NVLink;
    ``"disk"`` writes an HF safetensors export the engine reloads; ``"auto"``
    picks device when every engine is on this node.
    """

    role: ClassVar[str] = "training"
    service_cls: ClassVar[str] = "meshy_b200.service.training:TrainingService"
    endpoint_port_base: ClassVar[int] = 31000
    dist_port_base: ClassVar[int] = 41000

    model_path: str
    trainer_config: TrainerConfig
    batch_size: int
    trainer_params: TrainerParamsConfig | None = None
    timer_enabled: bool = True
    weight_sync_mode: Literal["disk", "device", "auto"] = "auto"
    weights_keep_latest_k: int = 5
    stream_minibatch: bool = False
    tq_endpoints_file: str | None = None
    partition_id: str = DEFAULT_DATA_PARTITION
    tq_fields: list[str] = field(default_factory=lambda: list(GRPO_TRAINER_FIELDS))
    tq_poll_interval: float = 0.5
    critic_cold_start_windows: int = 0
    checkpoint: GlobalCheckpointConfig = field(default_factory=GlobalCheckpointConfig)


@dataclass
class RolloutServiceConfig(ServiceConfig):
    """The CPU rollout driver (reference ``meshy/config.py:315-368``)."""

    role: ClassVar[str] = "rollout"
    service_cls: ClassVar[str] = "meshy_b200.service.rollout:RolloutService"
    uses_gpu: ClassVar[bool] = False

    model_path: str
    dataset: str
    dataset_kwargs: dict[str, Any] = field(default_factory=dict)
    reward: str | Callable[[Any], float] | None = None
    reward_shaping: str | Callable[..., float] | None = None
    reward_shaping_kwargs: dict[str, Any] = field(default_factory=dict)
    advantage: str | Callable[[list[Any]], Any] | None = None
    advantage_kwargs: dict[str, Any] = field(default_factory=dict)
    filter_zero_std_groups: bool = False
    publish_positive_lm_weights: bool = False
    oversample_factor: float = 1.0
    sampling_params: dict[str, Any] = field(default_factory=dict)
    group_size: int = 1
    num_epochs: int = 1
    poll_interval: float = 2.0
    async_max_running_request: int = -1
    pacing_window: int | str | None = "auto"
    tq_endpoints_file: str | None = None
    partition_id: str = DEFAULT_DATA_PARTITION
    verbose_trajectory_log: bool = False
    trajectory_log: str | None = None
    checkpoint: GlobalCheckpointConfig = field(default_factory=GlobalCheckpointConfig)
    external_advantage: bool = False

    def __post_init__(self) -> None:
        if self.oversample_factor < 1.0:
            raise ValueError(f"oversample_factor must be >= 1, got {self.oversample_factor!r}")
        if self.reward_shaping is not None and self.reward is None:
            raise ValueError("reward_shaping needs a reward to shape")
        if self.external_advantage and self.advantage is not None:
            raise ValueError("external_advantage and advantage are mutually exclusive")


# ── PPO critic (VAPO-GAE advantage) ─────────────────────────────────────
CRITIC_INPUT_FIELDS = ["tokens", "mask_assistant", "reward", "weight_version"]
CRITIC_OUTPUT_FIELDS_BY_MODE = {
    "values": ["values"],
    "advantage": ["advantage"],
}
CRITIC_OUTPUT_FIELDS = CRITIC_OUTPUT_FIELDS_BY_MODE["advantage"]
GAE_TRAINER_FIELDS = [f for f in GRPO_TRAINER_FIELDS if f != "advantage"] + ["values"]
GAE_TRAINER_FIELDS_SHAPED = GAE_TRAINER_FIELDS + ["raw_reward"]


@dataclass
class CriticServiceConfig(ServiceConfig):
    """Independent value-net replica (reference ``meshy/config.py:407-496``)."""

    role: ClassVar[str] = "critic"
    service_cls: ClassVar[str] = "meshy_b200.service.critic:CriticService"
    endpoint_port_base: ClassVar[int] = 33000
    dist_port_base: ClassVar[int] = 43000

    model_path: str
    trainer_config: TrainerConfig
    score_batch_size: int
    publish_mode: Literal["values", "advantage"] = "values"
    micro_rows: int = 1
    max_tokens_per_micro: int | None = None
    train_backbone: bool = True
    lr: float = 5e-6
    optimizer_kwargs: dict[str, Any] | None = None
    value_clip: float | None = None
    warmup_steps: int = 10
    cold_start_windows: int = 30
    publish_gate_zero: bool = False
    value_epochs: int = 1
    gamma: float = 1.0
    alpha: float = 1.5
    max_norm: float = 1.0
    timer_enabled: bool = True
    tq_endpoints_file: str | None = None
    partition_id: str = DEFAULT_DATA_PARTITION
    tq_poll_interval: float = 0.5
    checkpoint: GlobalCheckpointConfig = field(default_factory=GlobalCheckpointConfig)

    def __post_init__(self) -> None:
        if self.publish_mode not in CRITIC_OUTPUT_FIELDS_BY_MODE:
            raise ValueError(
                f"publish_mode must be one of {sorted(CRITIC_OUTPUT_FIELDS_BY_MODE)}, got {self.publish_mode!r}"
            )
        if self.micro_rows <= 0:
            raise ValueError("micro_rows must be positive")

    @property
    def output_fields(self) -> list[str]:
        return list(CRITIC_OUTPUT_FIELDS_BY_MODE[self.publish_mode])


# ── Student Top-K on-policy distillation (OPD) ──────────────────────────
OPD_TEACHER_FIELDS = ["teacher_topk_ids", "teacher_topk_logprobs"]
OPD_TRAINER_FIELDS = GRPO_TRAINER_FIELDS + OPD_TEACHER_FIELDS


@dataclass
class OPDTeacherConfig(ServiceConfig):
    """Frozen teacher that appends Top-K log-prob columns to rollout rows."""

    role: ClassVar[str] = "teacher"
    service_cls: ClassVar[str] = "meshy_b200.service.opd:OPDTeacherService"
    endpoint_port_base: ClassVar[int] = 32000
    dist_port_base: ClassVar[int] = 42000

    model_path: str
    trainer_config: TrainerConfig
    top_k: int = 8
    score_batch_size: int = 8
    student_group: str | None = None
    tq_endpoints_file: str | None = None
    partition_id: str = DEFAULT_DATA_PARTITION
    tq_poll_interval: float = 0.5
    timer_enabled: bool = False

    def __post_init__(self) -> None:
        if self.top_k <= 0:
            raise ValueError("OPDTeacherConfig.top_k must be positive")
        if self.score_batch_size <= 0:
            raise ValueError("OPDTeacherConfig.score_batch_size must be positive")
        if self.trainer_config.cp_degree != 1:
            raise ValueError("the OPD Teacher does not support context parallelism yet")


@dataclass
class OPDTrainingConfig(TrainingServiceConfig):
    """Student trainer: the ordinary training service with the Top-K KL loss."""

    service_cls: ClassVar[str] = "meshy_b200.service.opd:OPDTrainingService"

    tq_fields: list[str] = field(default_factory=lambda: list(OPD_TRAINER_FIELDS))
    log_prob_min_clamp: float | None = -10.0
    loss_max_clamp: float | None = 10.0


__all__ = [
    "CRITIC_INPUT_FIELDS",
    "CRITIC_OUTPUT_FIELDS",
    "CRITIC_OUTPUT_FIELDS_BY_MODE",
    "CriticServiceConfig",
    "DEFAULT_DATA_PARTITION",
    "GAE_TRAINER_FIELDS",
    "GAE_TRAINER_FIELDS_SHAPED",
    "GRPO_TRAINER_FIELDS",
    "GlobalCheckpointConfig",
    "InferenceServiceConfig",
    "OPDTeacherConfig",
    "OPDTrainingConfig",
    "OPD_TEACHER_FIELDS",
    "OPD_TRAINER_FIELDS",
    "RolloutServiceConfig",
    "SamplingParams",
    "ServiceConfig",
    "TrainerConfig",
    "TrainerParamsConfig",
    "TrainingServiceConfig",
]

"""Experimental (``dev``) configuration TypedDicts.

Covers the knobs of the reference's ``src/art/dev/train.py:11-50`` (the loss
and data knobs of ``dev.TrainConfig``), ``src/art/dev/model.py`` (LoRA,
engine and internal model config) and ``src/art/dev/openai_server.py``.
Everything is optional; absent keys take the documented defaults at use sites.
"""

from __future__ import annotations

from typing import Any, Literal

from typing_extensions import TypedDict


class TrainConfig(TypedDict, total=False):
    """Loss / data knobs consumed by the GRPO step and the packer."""

    advantage_balance: float
    allow_training_without_logprobs: bool
    epsilon: float
    epsilon_high: float | None
    importance_sampling_level: Literal[
        "token", "sequence", "average", "geometric_average"
    ]
    kimi_k2_tau: float | None
    kl_penalty_coef: float
    kl_penalty_reference_step: int | None
    kl_penalty_source: Literal["current_learner", "sample"]
    kl_penalty_step_lag: int | None
    kl_ref_adapter_path: str | None
    logprob_calculation_chunk_size: int
    mask_prob_ratio: bool
    max_negative_advantage_importance_sampling_weight: float
    moe_routing_replay_bundle: Any
    moe_routing_replay_path: str | None
    moe_routing_replay_strict: bool
    num_trajectories_learning_rate_multiplier_power: float
    packed_sequence_length: int | None
    plot_tensors: bool
    ppo: bool
    precalculate_logprobs: bool
    scale_learning_rate_by_reward_std_dev: bool
    scale_rewards: bool
    truncated_importance_sampling: float | None


class TrainSFTConfig(TypedDict, total=False):
    metric_logging: dict[str, Any]


class LoRAConfig(TypedDict, total=False):
    """LoRA adapter shape (PEFT ``LoraConfig`` field names)."""

    r: int
    lora_alpha: int
    target_modules: list[str]
    lora_dropout: float
    bias: str


class InitArgs(TypedDict, total=False):
    max_seq_length: int
    dtype: str
    seed: int


class TrainerArgs(TypedDict, total=False):
    learning_rate: float
    adam_beta1: float
    adam_beta2: float
    adam_epsilon: float
    weight_decay: float
    max_grad_norm: float
    optim: str


class EngineArgs(TypedDict, total=False):
    """Rollout-engine arguments forwarded to the inference server."""

    gpu_memory_utilization: float
    max_model_len: int
    enable_lora: bool
    max_lora_rank: int
    tensor_parallel_size: int
    enable_sleep_mode: bool


class OpenAIServerConfig(TypedDict, total=False):
    host: str
    port: int
    log_file: str
    server_args: dict[str, Any]
    engine_args: EngineArgs


class InternalModelConfig(TypedDict, total=False):
    """Backend-specific model configuration (``TrainableModel._internal_config``)."""

    init_args: InitArgs
    engine_args: EngineArgs
    peft_args: LoRAConfig
    trainer_args: TrainerArgs
    trainer_gpu_ids: list[int]
    inference_gpu_ids: list[int]
    rollout_weights_mode: Literal["lora", "merged"]
    chat_template: str
    chat_template_kwargs: dict[str, Any]
    model_preset: str
    topology: dict[str, int]


DEFAULT_LORA_TARGETS = [
    "q_proj",
    "k_proj",
    "v_proj",
    "o_proj",
    "gate_proj",
    "up_proj",
    "down_proj",
]


def default_lora_config(r: int = 8, alpha: int = 16) -> LoRAConfig:
    return LoRAConfig(
        r=r, lora_alpha=alpha, target_modules=list(DEFAULT_LORA_TARGETS), lora_dropout=0.0
    )


def default_trainer_args() -> TrainerArgs:
    """Optimizer defaults of the reference (``dev/get_model_config.py:78-95``):
    lr 5e-6, betas (0.9, 0.99), weight decay 0.1, grad clip 0.1."""
    return TrainerArgs(
        learning_rate=5e-6,
        adam_beta1=0.9,
        adam_beta2=0.99,
        adam_epsilon=1e-8,
        weight_decay=0.1,
        max_grad_norm=0.1,
        optim="adamw",
    )


def validate_dedicated_config(config: InternalModelConfig) -> None:
    """Dedicated mode (separate trainer / inference GPUs) must name disjoint
    GPU sets (reference ``dev/validate.py:37-118``)."""
    trainer = config.get("trainer_gpu_ids")
    inference = config.get("inference_gpu_ids")
    if trainer is None and inference is None:
        return
    if not trainer or not inference:
        raise ValueError(
            "dedicated mode needs both trainer_gpu_ids and inference_gpu_ids"
        )
    if set(trainer) & set(inference):
        raise ValueError("trainer_gpu_ids and inference_gpu_ids must not overlap")
    if config.get("rollout_weights_mode", "lora") not in ("lora", "merged"):
        raise ValueError("rollout_weights_mode must be 'lora' or 'merged'")

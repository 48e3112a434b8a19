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
    model_name: str


class TrainerArgs(TypedDict, total=False):
    learning_rate: float
    adam_beta1: float
    adam_beta2: float
    adam_epsilon: float
    weight_decay: float
    max_grad_norm: float
    optim: str


class EngineArgs(TypedDict, total=False):
    """Rollout-engine arguments.  The native engine reads ``max_model_len``
    (KV-cache length per sequence), ``max_num_seqs`` (sequences decoded per
    batch) and ``max_lora_rank``; ``enable_sleep_mode`` is False in
    dedicated mode (the engine owns its GPUs).  The other keys are kept for
    configs shared with a vLLM server."""

    gpu_memory_utilization: float
    max_model_len: int
    max_num_seqs: int
    enable_lora: bool
    max_lora_rank: int
    tensor_parallel_size: int
    enable_sleep_mode: bool
    lora_target_modules: list[str]
    generation_config: str


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


class BackendModelConfig(TypedDict, total=False):
    """Fully resolved model configuration of a backend (defaults merged with
    the user's ``_internal_config``)."""

    init_args: InitArgs
    engine_args: EngineArgs
    lora_config: LoRAConfig
    trainer_args: TrainerArgs
    rollout_weights_mode: Literal["lora", "merged"]
    trainer_gpu_ids: list[int]
    inference_gpu_ids: list[int]
    allow_unvalidated_arch: bool


def is_dedicated_mode(config: InternalModelConfig) -> bool:
    """Separate trainer and inference GPUs (both id lists given)."""
    return bool(config.get("trainer_gpu_ids")) and bool(config.get("inference_gpu_ids"))


def get_model_config(base_model: str, output_dir: str, config: InternalModelConfig | None,
                     lora_config: LoRAConfig | None = None) -> BackendModelConfig:
    """Defaults merged with ``config`` (reference ``dev/get_model_config.py:22-113``):

    * ``init_args``: ``max_seq_length`` = the architecture's context length,
      the model to load = the latest checkpoint under ``output_dir`` if any;
    * ``engine_args``: ``max_model_len`` = ``max_seq_length``, 256 sequences
      per decode batch, sleep mode only when sharing GPUs with the trainer,
      LoRA targets of the family;
    * ``lora_config``: the family's default target modules (model-support
      registry), r 8, alpha 16;
    * ``trainer_args``: AdamW lr 5e-6, betas (0.9, 0.99), weight decay 0.1,
      grad clip 0.1, constant schedule.
    User values override every default key by key.
    """
    import os

    from .models.config import get_config
    from .models.registry import get_model_support
    from .utils.output_dirs import get_step_checkpoint_dir, list_checkpoint_steps

    config = dict(config or {})
    validate_dedicated_config(config)  # type: ignore[arg-type]
    dedicated = is_dedicated_mode(config)  # type: ignore[arg-type]
    try:
        mcfg = get_config(config.get("model_preset") or base_model)
        max_len = int(min(mcfg.max_position_embeddings, 32768))
        targets = list(get_model_support(mcfg, allow_unvalidated_arch=True).default_target_modules)
    except KeyError:
        max_len, targets = 8192, list(DEFAULT_LORA_TARGETS)
    init = InitArgs(max_seq_length=max_len)
    init.update(config.get("init_args") or {})
    model_name = base_model
    steps = list_checkpoint_steps(output_dir) if output_dir and os.path.isdir(output_dir) else []
    if steps:
        model_name = get_step_checkpoint_dir(output_dir, max(steps))
    engine = EngineArgs(max_model_len=int(init.get("max_seq_length", max_len)), max_num_seqs=256,
                        enable_sleep_mode=not dedicated, generation_config="vllm")
    engine.update(config.get("engine_args") or {})
    if dedicated:
        engine["enable_sleep_mode"] = False
    lora = LoRAConfig(r=8, lora_alpha=16, target_modules=targets, lora_dropout=0.0)
    lora.update(config.get("peft_args") or {})
    lora.update(lora_config or {})
    mode = config.get("rollout_weights_mode", "lora")
    if mode == "lora":
        engine.setdefault("lora_target_modules", list(lora["target_modules"]))
        engine.setdefault("max_lora_rank", int(lora["r"]))
    trainer = default_trainer_args()
    trainer.update(config.get("trainer_args") or {})
    out = BackendModelConfig(init_args=init, engine_args=engine, lora_config=lora, trainer_args=trainer,
                             rollout_weights_mode=mode)
    out["init_args"]["model_name"] = model_name  # type: ignore[typeddict-unknown-key]
    for key in ("trainer_gpu_ids", "inference_gpu_ids", "allow_unvalidated_arch"):
        if key in config:
            out[key] = config[key]  # type: ignore[literal-required]
    return out

"""The contract every backend implements (reference ``src/art/backend.py:15-52``)
and the shared mapping of ``train()`` keyword arguments onto the stable and
experimental training configs (reference ``src/art/_backend_training.py:15-111``)."""

from __future__ import annotations

from typing import TYPE_CHECKING, Any, AsyncIterator, Iterable, Literal, Protocol

from . import dev
from .trajectories import Trajectory, TrajectoryGroup
from .types import TrainConfig, TrainResult, TrainSFTConfig

if TYPE_CHECKING:
    from .model import Model, TrainableModel


class Backend(Protocol):
    def _model_inference_name(self, model: "Model", step: int | None = None) -> str: ...

    async def close(self) -> None: ...

    async def register(self, model: "Model") -> None: ...

    async def _get_step(self, model: "TrainableModel") -> int: ...

    async def _delete_checkpoint_files(self, model: "TrainableModel", steps_to_keep: list[int]) -> None: ...

    async def _prepare_backend_for_training(
        self, model: "TrainableModel", config: dev.OpenAIServerConfig | None
    ) -> tuple[str, str]: ...

    async def train(
        self, model: "TrainableModel", trajectory_groups: Iterable[TrajectoryGroup], **kwargs: Any
    ) -> TrainResult: ...

    def _train_sft(
        self,
        model: "TrainableModel",
        trajectories: Iterable[Trajectory],
        config: TrainSFTConfig,
        dev_config: dev.TrainSFTConfig,
        verbose: bool = False,
    ) -> AsyncIterator[dict[str, float]]: ...


def build_rl_train_configs(
    *,
    learning_rate: float,
    advantage_balance: float = 0.0,
    scale_rewards: bool = True,
    importance_sampling_level: Literal["token", "sequence", "average", "geometric_average"] = "token",
    mask_prob_ratio: bool = False,
    ppo: bool = False,
    precalculate_logprobs: bool = False,
    epsilon: float | None = None,
    epsilon_high: float | None = None,
    max_negative_advantage_importance_sampling_weight: float | None = None,
    kimi_k2_tau: float | None = None,
    kl_penalty_coef: float = 0.0,
    kl_penalty_source: Literal["current_learner", "sample"] = "current_learner",
    allow_training_without_logprobs: bool | None = None,
    plot_tensors: bool | None = None,
    truncated_importance_sampling: float | None = None,
    scale_learning_rate_by_reward_std_dev: bool | None = None,
    logprob_calculation_chunk_size: int | None = None,
    packed_sequence_length: int | None = None,
    num_trajectories_learning_rate_multiplier_power: float | None = None,
    kl_ref_adapter_path: str | None = None,
) -> tuple[TrainConfig, dev.TrainConfig]:
    config = TrainConfig(
        learning_rate=learning_rate, kl_penalty_coef=kl_penalty_coef, kl_penalty_source=kl_penalty_source
    )
    d: dict[str, Any] = {
        "advantage_balance": advantage_balance,
        "importance_sampling_level": importance_sampling_level,
        "kl_penalty_coef": kl_penalty_coef,
        "kl_penalty_source": kl_penalty_source,
        "mask_prob_ratio": mask_prob_ratio,
        "ppo": ppo,
        "precalculate_logprobs": precalculate_logprobs,
        "scale_rewards": scale_rewards,
    }
    optional = {
        "allow_training_without_logprobs": allow_training_without_logprobs,
        "plot_tensors": plot_tensors,
        "truncated_importance_sampling": truncated_importance_sampling,
        "scale_learning_rate_by_reward_std_dev": scale_learning_rate_by_reward_std_dev,
        "logprob_calculation_chunk_size": logprob_calculation_chunk_size,
        "packed_sequence_length": packed_sequence_length,
        "num_trajectories_learning_rate_multiplier_power": num_trajectories_learning_rate_multiplier_power,
        "epsilon": epsilon,
        "epsilon_high": epsilon_high,
        "max_negative_advantage_importance_sampling_weight": max_negative_advantage_importance_sampling_weight,
        "kimi_k2_tau": kimi_k2_tau,
        "kl_ref_adapter_path": kl_ref_adapter_path,
    }
    d.update({k: v for k, v in optional.items() if v is not None})
    return config, d  # type: ignore[return-value]


def aggregate_rl_training_metrics(
    training_metrics: list[dict[str, float]], trajectory_groups: Iterable[TrajectoryGroup]
) -> dict[str, float]:
    """Average per-step metric dicts and add group summary statistics."""
    from .metrics import summarize_groups

    out: dict[str, float] = {}
    keys = {k for m in training_metrics for k in m}
    for k in keys:
        vals = [m[k] for m in training_metrics if k in m]
        out[k] = sum(vals) / len(vals)
    for k, v in summarize_groups(list(trajectory_groups)).items():
        out.setdefault(f"train/{k}", v)
    return out

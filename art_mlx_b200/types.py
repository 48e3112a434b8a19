"""Public configuration and result types.

Mirrors the public pydantic/dataclass surface of the reference
(``src/art/types.py:26-106``): ``TrainConfig``, ``TrainSFTConfig``,
``MegatronTopologyConfig`` (here ``TopologyConfig`` with a compatible alias),
``MegatronRuntimeConfig`` and the ``TrainResult`` family.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Annotated, Any, Literal

import pydantic
from pydantic import SkipValidation
from typing_extensions import TypedDict

try:  # the OpenAI wire types are the rollout format; keep them optional on import
    from openai.types.chat.chat_completion import Choice as Choice
    from openai.types.chat.chat_completion_message_param import (
        ChatCompletionMessageParam,
    )
    from openai.types.chat.chat_completion_tool_param import ChatCompletionToolParam
except Exception:  # pragma: no cover - openai is part of the image
    Choice = Any  # type: ignore[misc,assignment]
    ChatCompletionMessageParam = dict  # type: ignore[misc,assignment]
    ChatCompletionToolParam = dict  # type: ignore[misc,assignment]

Message = Annotated[ChatCompletionMessageParam, SkipValidation]
MessageOrChoice = Message | Choice
Messages = list[Message]
MessagesAndChoices = list[MessageOrChoice]
Tools = list[ChatCompletionToolParam]

Verbosity = Literal[0, 1, 2]


def visible_device_count() -> int:
    """Number of visible CUDA devices, at least 1 (CPU hosts report 1)."""
    try:
        import torch

        return max(int(torch.cuda.device_count()), 1)
    except Exception:
        return 1


class TrainConfig(pydantic.BaseModel):
    """Per-call RL training knobs (reference ``types.py:26-30``)."""

    learning_rate: float = 5e-6
    kl_penalty_coef: float = 0.0
    kl_penalty_source: Literal["current_learner", "sample"] = "current_learner"
    grad_accumulation_sequences: int | None = pydantic.Field(default=None, ge=1)


class TopologyConfig(pydantic.BaseModel):
    """Parallel topology of the trainer.

    Same fields and defaults as the reference's ``MegatronTopologyConfig``
    (``types.py:33-39``): ``cp`` and ``ep`` default to every visible GPU.
    ``dp`` is derived: ``world / (tp * cp * pp)``.
    """

    tp: int = pydantic.Field(default=1, ge=1)
    cp: int = pydantic.Field(default_factory=visible_device_count, ge=1)
    ep: int = pydantic.Field(default_factory=visible_device_count, ge=1)
    pp: int = pydantic.Field(default=1, ge=1)
    vpp: int | None = pydantic.Field(default=None, ge=1)
    etp: int = pydantic.Field(default=1, ge=1)

    def data_parallel_size(self, world_size: int) -> int:
        denom = self.tp * self.cp * self.pp
        if world_size % denom != 0:
            raise ValueError(
                f"world size {world_size} is not divisible by tp*cp*pp={denom}"
            )
        return world_size // denom


MegatronTopologyConfig = TopologyConfig


class RuntimeConfig(pydantic.BaseModel):
    """Frozen runtime configuration (reference ``types.py:42-46``)."""

    model_config = pydantic.ConfigDict(frozen=True)

    topology: TopologyConfig
    packed_sequence_length: int = pydantic.Field(ge=1)


MegatronRuntimeConfig = RuntimeConfig


class TrainSFTConfig(pydantic.BaseModel):
    """Supervised fine-tuning knobs (reference ``types.py:49-53``)."""

    learning_rate: float | list[float] = 5e-5
    batch_size: int | Literal["auto"] = "auto"
    assistant_turns: Literal["all", "last"] = "all"


class SFTMetricLoggingConfig(TypedDict, total=False):
    enabled: bool
    target_training_step: int


@dataclass
class TrainResult:
    """Result of ``backend.train()``: the step reached and averaged metrics."""

    step: int
    metrics: dict[str, float] = field(default_factory=dict)


@dataclass
class LocalTrainResult(TrainResult):
    """Result of ``LocalBackend.train()``; adds the saved checkpoint directory."""

    checkpoint_path: str | None = None


@dataclass
class ServerlessTrainResult(TrainResult):
    """Result shape of a remote (artifact-backed) backend."""

    artifact_name: str | None = None

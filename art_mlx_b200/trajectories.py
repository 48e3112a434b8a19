"""Rollout data model: ``Trajectory``, ``TrajectoryGroup``, ``History``.

Behaviour follows the reference ``src/art/trajectories.py:30-319``:
a trajectory is a list of chat messages and sampled ``Choice`` objects plus a
scalar reward; a group collects the trajectories sampled for one prompt and
is the unit of GRPO advantage normalisation.  A group built from awaitables
is itself awaitable (it resolves the rollouts concurrently, recording
exceptions within the active gather context's budget).
"""

from __future__ import annotations

import asyncio
import copy
import time
import traceback
from contextlib import asynccontextmanager
from datetime import datetime
from typing import Any, AsyncGenerator, Awaitable, Iterable, Iterator, cast

import pydantic

from .types import Choice, Messages, MessagesAndChoices, Tools

MetadataValue = float | int | str | bool | None


class PydanticException(pydantic.BaseModel):
    type: str
    message: str
    traceback: str

    @classmethod
    def from_exception(cls, exc: BaseException) -> "PydanticException":
        return cls(
            type=str(type(exc)),
            message=str(exc),
            traceback="\n".join(
                traceback.format_exception(type(exc), exc, exc.__traceback__)
            ),
        )


def _is_choice(item: Any) -> bool:
    return not isinstance(item, dict) and hasattr(item, "message") and hasattr(
        item, "finish_reason"
    )


def get_messages(messages_and_choices: MessagesAndChoices) -> Messages:
    """Flatten messages and choices into plain chat messages (choices become
    assistant messages, with tool calls when present)."""
    out: Messages = []
    for item in messages_and_choices:
        if _is_choice(item):
            msg = item.message  # type: ignore[union-attr]
            entry: dict[str, Any] = {"role": "assistant", "content": msg.content or ""}
            if msg.tool_calls:
                entry["tool_calls"] = [
                    call.model_dump(mode="json") for call in msg.tool_calls
                ]
            out.append(cast(Any, entry))
        else:
            entry = dict(item)  # type: ignore[arg-type]
            if entry.get("content") is None:
                entry["content"] = ""
            out.append(cast(Any, entry))
    return out


class History(pydantic.BaseModel):
    messages_and_choices: MessagesAndChoices
    tools: Tools | None = None

    def messages(self) -> Messages:
        return get_messages(self.messages_and_choices)


class Trajectory(pydantic.BaseModel):
    messages_and_choices: MessagesAndChoices = []
    tools: Tools | None = None
    additional_histories: list[History] = []
    reward: float = 0.0
    initial_policy_version: int | None = None
    final_policy_version: int | None = None
    metrics: dict[str, float | int | bool] = {}
    metadata: dict[str, MetadataValue] = {}
    logs: list[str] = []
    start_time: datetime = pydantic.Field(default_factory=datetime.now, exclude=True)

    def log(self, message: str) -> None:
        self.logs.append(message)

    def finish(self) -> "Trajectory":
        self.metrics["duration"] = (datetime.now() - self.start_time).total_seconds()
        return self

    @asynccontextmanager
    async def track_duration(self, metric_name: str) -> AsyncGenerator[None, None]:
        started = time.monotonic()
        try:
            yield
        finally:
            key = f"{metric_name}_duration"
            self.metrics[key] = self.metrics.get(key, 0.0) + (time.monotonic() - started)

    def __str__(self) -> str:
        return (
            f"Trajectory(reward={self.reward}, metrics={self.metrics}, "
            f"metadata={self.metadata})"
        )

    def messages(self) -> Messages:
        return get_messages(self.messages_and_choices)

    def for_logging(self) -> dict[str, Any]:
        messages = []
        for item in self.messages_and_choices:
            if _is_choice(item):
                messages.append({**item.message.to_dict(), "trainable": True})  # type: ignore[union-attr]
            else:
                messages.append({**dict(item), "trainable": False})  # type: ignore[arg-type]
        return {
            "reward": self.reward,
            "initial_policy_version": self.initial_policy_version,
            "final_policy_version": self.final_policy_version,
            "metrics": self.metrics,
            "metadata": self.metadata,
            "messages": messages,
            "tools": self.tools,
            "logs": self.logs,
        }


class _AwaitableGroup:
    """Awaitable returned when a group is built from rollout coroutines."""

    def __init__(self, coro: Any, num_trajectories: int) -> None:
        self._coro = coro
        self._num_trajectories = num_trajectories

    def __await__(self):
        return self._coro.__await__()


class TrajectoryGroup(pydantic.BaseModel):
    trajectories: list[Trajectory]
    exceptions: list[PydanticException] = []
    metadata: dict[str, MetadataValue] = {}
    metrics: dict[str, float | int | bool] = {}
    logs: list[str] = []

    def __new__(cls, trajectories: Iterable[Any] = (), **kwargs: Any):  # type: ignore[misc]
        items = list(trajectories)
        if any(hasattr(item, "__await__") for item in items):
            return _AwaitableGroup(
                cls._resolve(
                    items,
                    list(kwargs.get("exceptions") or []),
                    kwargs.get("metadata"),
                    kwargs.get("metrics"),
                    kwargs.get("logs"),
                ),
                len(items),
            )
        instance = super().__new__(cls)
        instance._pending_items = items  # consumed by __init__
        return instance

    def __init__(
        self,
        trajectories: Iterable[Any] = (),
        *,
        exceptions: list[BaseException] | None = None,
        metadata: dict[str, MetadataValue] | None = None,
        metrics: dict[str, float | int | bool] | None = None,
        logs: list[str] | None = None,
    ) -> None:
        items = self.__dict__.pop("_pending_items", None)
        if items is None:
            items = list(trajectories)
        trajs = [t for t in items if isinstance(t, Trajectory)]
        errors = [e for e in items if isinstance(e, BaseException)] + list(
            exceptions or []
        )
        super().__init__(
            trajectories=trajs,
            exceptions=[
                e if isinstance(e, PydanticException) else PydanticException.from_exception(e)
                for e in errors
            ],
            metadata=metadata or {},
            metrics=metrics or {},
            logs=logs or [],
        )

    def __setattr__(self, name: str, value: Any) -> None:
        if name == "_pending_items":
            object.__setattr__(self, name, value)
            return
        super().__setattr__(name, value)

    @staticmethod
    async def _resolve(
        items: list[Any],
        exceptions: list[BaseException],
        metadata: dict[str, MetadataValue] | None,
        metrics: dict[str, float | int | bool] | None,
        logs: list[str] | None,
    ) -> "TrajectoryGroup":
        from .gather import get_gather_context, record_metrics

        context = get_gather_context()
        done: list[Trajectory] = []
        for future in asyncio.as_completed(cast(list[Awaitable[Trajectory]], items)):
            try:
                trajectory = await future
            except BaseException as exc:  # noqa: BLE001 - budgeted by the context
                exceptions.append(exc)
                context.metric_sums["exceptions"] += 1
                context.update_pbar(n=0)
                if context.too_many_exceptions():
                    raise
                continue
            done.append(trajectory)
            record_metrics(context, trajectory)
            context.update_pbar(n=1)
        return TrajectoryGroup(
            done, exceptions=exceptions, metadata=metadata, metrics=metrics, logs=logs
        )

    def log(self, message: str) -> None:
        self.logs.append(message)

    def __iter__(self) -> Iterator[Trajectory]:  # type: ignore[override]
        return iter(self.trajectories)

    def __len__(self) -> int:
        return len(self.trajectories)

    def __copy__(self) -> "TrajectoryGroup":
        new = TrajectoryGroup(
            self.trajectories[:],
            metadata=dict(self.metadata),
            metrics=dict(self.metrics),
            logs=self.logs[:],
        )
        new.exceptions = self.exceptions[:]
        return new

    def __deepcopy__(self, memo: dict[int, Any] | None = None) -> "TrajectoryGroup":
        memo = {} if memo is None else memo
        if id(self) in memo:
            return memo[id(self)]
        new = TrajectoryGroup(
            copy.deepcopy(self.trajectories, memo),
            metadata=copy.deepcopy(self.metadata, memo),
            metrics=copy.deepcopy(self.metrics, memo),
            logs=copy.deepcopy(self.logs, memo),
        )
        memo[id(self)] = new
        new.exceptions = copy.deepcopy(self.exceptions, memo)
        return new

"""``Model`` / ``TrainableModel``: the user-facing model handles.

Public surface of the reference ``src/art/model.py:166-1353``:

* ``Model(name, project, inference_api_key, inference_base_url, ...)`` for
  prompted / comparison models; ``TrainableModel(name, project, base_model,
  lora_config, _internal_config)`` for trained ones;
* ``await model.register(backend)`` → the backend prepares training and
  inference and fills ``inference_base_url`` / ``inference_api_key`` /
  ``inference_model_name`` (``name@step``);
* ``model.openai_client()`` → an ``AsyncOpenAI`` whose chat completions ask
  the rollout server for token ids (``return_token_ids``) and attach
  ``prompt_token_ids`` / ``token_ids`` to every returned ``Choice``, which is
  what training consumes;
* ``await model.log(groups | metrics, split, step)`` → ``history.jsonl`` and
  per-step parquet trajectories; ``get_step``; ``delete_checkpoints``;
  ``train_sft``; JSON ``state`` helpers.
"""

from __future__ import annotations

import json
import os
import time
from typing import TYPE_CHECKING, Any, AsyncIterator, Generic, Iterable, TypeVar

import pydantic
from pydantic import BaseModel

from . import dev
from .trajectories import Trajectory, TrajectoryGroup
from .types import TrainSFTConfig

if TYPE_CHECKING:
    from .backend import Backend

ModelConfig = TypeVar("ModelConfig", bound=BaseModel | None)
StateType = TypeVar("StateType", bound=dict[str, Any])


def _attach_token_ids(response: Any) -> None:
    """Copy server-returned token ids from the raw payload onto each Choice."""
    from .preprocessing.tokenize import attach_token_ids_to_choice

    payload = getattr(response, "model_extra", None) or {}
    raw = {"prompt_token_ids": payload.get("prompt_token_ids"), "choices": []}
    for choice in getattr(response, "choices", []) or []:
        extra = getattr(choice, "model_extra", None) or {}
        raw["choices"].append({"token_ids": extra.get("token_ids"), "routed_experts": extra.get("routed_experts")})
    for i, choice in enumerate(getattr(response, "choices", []) or []):
        attach_token_ids_to_choice(choice, raw, i)


class _ChatCompletions:
    def __init__(self, inner: Any, extra_body: dict[str, Any] | None) -> None:
        self._inner = inner
        self._extra = extra_body

    async def create(self, *args: Any, **kwargs: Any) -> Any:
        if self._extra:
            body = dict(self._extra)
            body.update(kwargs.get("extra_body") or {})
            kwargs["extra_body"] = body
        response = await self._inner.create(*args, **kwargs)
        if not kwargs.get("stream"):
            _attach_token_ids(response)
        return response

    def __getattr__(self, name: str) -> Any:
        return getattr(self._inner, name)


class _Chat:
    def __init__(self, inner: Any, extra_body: dict[str, Any] | None) -> None:
        self._inner = inner
        self.completions = _ChatCompletions(inner.completions, extra_body)

    def __getattr__(self, name: str) -> Any:
        return getattr(self._inner, name)


class _ClientProxy:
    def __init__(self, client: Any, extra_body: dict[str, Any] | None) -> None:
        self._client = client
        self._extra = extra_body
        self.chat = _Chat(client.chat, extra_body)

    def with_options(self, *args: Any, **kwargs: Any) -> "_ClientProxy":
        return _ClientProxy(self._client.with_options(*args, **kwargs), self._extra)

    def __getattr__(self, name: str) -> Any:
        return getattr(self._client, name)


class Model(BaseModel, Generic[ModelConfig, StateType]):
    model_config = pydantic.ConfigDict(arbitrary_types_allowed=True)

    name: str
    project: str
    entity: str | None = None
    id: str | None = None
    run_id: str | None = None
    config: Any = None
    trainable: bool = False
    inference_api_key: str | None = None
    inference_base_url: str | None = None
    inference_model_name: str | None = None
    base_path: str = ".art"
    report_metrics: list[str] | None = None

    _backend: Any = pydantic.PrivateAttr(default=None)
    _openai_client: Any = pydantic.PrivateAttr(default=None)

    def backend(self) -> "Backend":
        if self._backend is None:
            raise ValueError("Model is not registered with a backend; call `await model.register(backend)`")
        return self._backend

    async def register(self, backend: "Backend") -> None:
        if self.config is not None:
            try:
                json.dumps(self.config.model_dump() if hasattr(self.config, "model_dump") else self.config)
            except Exception as exc:
                raise ValueError("The model config cannot be serialized to JSON") from exc
        self._backend = backend
        await backend.register(self)

    def _default_extra_body(self) -> dict[str, Any] | None:
        body: dict[str, Any] = {}
        if self.trainable:
            body["return_token_ids"] = True
            body["return_tokens_as_token_ids"] = True
        internal = getattr(self, "_internal_config", None) or {}
        if internal.get("chat_template_kwargs") is not None:
            body["chat_template_kwargs"] = dict(internal["chat_template_kwargs"])
        return body or None

    def openai_client(self) -> Any:
        if self._openai_client is not None:
            return self._openai_client
        if self.inference_api_key is None or self.inference_base_url is None:
            if self.trainable:
                raise ValueError("OpenAI client not available yet: call `model.register()` first")
            raise ValueError("provide `inference_api_key` and `inference_base_url`")
        from openai import AsyncOpenAI

        raw = AsyncOpenAI(base_url=self.inference_base_url, api_key=self.inference_api_key)
        self._openai_client = _ClientProxy(raw, self._default_extra_body())
        return self._openai_client

    def litellm_completion_params(self, step: int | None = None) -> dict[str, Any]:
        name = self.get_inference_name(step)
        if self.trainable:
            name = f"hosted_vllm/{name}"
        params: dict[str, Any] = {
            "model": name,
            "base_url": self.inference_base_url,
            "api_key": self.inference_api_key,
            "temperature": 1,
        }
        if extra := self._default_extra_body():
            params["extra_body"] = extra
        return params

    def get_inference_name(self, step: int | None = None) -> str:
        if self._backend is not None and hasattr(self._backend, "_model_inference_name"):
            return self._backend._model_inference_name(self, step=step)
        base = self.inference_model_name or self.name
        return f"{base}@{step}" if step is not None else base

    def _get_output_dir(self) -> str:
        return f"{self.base_path}/{self.project}/models/{self.name}"

    # ---- JSON state -----------------------------------------------------
    def _state_path(self) -> str:
        return os.path.join(self._get_output_dir(), "state.json")

    def read_state(self) -> StateType | None:
        try:
            with open(self._state_path()) as f:
                return json.load(f)
        except FileNotFoundError:
            return None

    def overwrite_state(self, state: StateType) -> None:
        os.makedirs(self._get_output_dir(), exist_ok=True)
        tmp = self._state_path() + ".tmp"
        with open(tmp, "w") as f:
            json.dump(state, f)
        os.replace(tmp, self._state_path())

    def write_state(self, state: StateType) -> None:
        self.overwrite_state(state)

    def merge_state(self, state: dict[str, Any]) -> StateType:
        merged = _deep_merge(self.read_state() or {}, state)
        self.overwrite_state(merged)  # type: ignore[arg-type]
        return merged  # type: ignore[return-value]

    # ---- logging ----------------------------------------------------------
    async def log(
        self,
        trajectories: Iterable[Trajectory | TrajectoryGroup] | None = None,
        split: str = "val",
        *,
        metrics: dict[str, float] | None = None,
        step: int | None = None,
    ) -> None:
        """Append metrics to ``history.jsonl`` and write the step's
        trajectories to ``trajectories/{split}/{step:04d}.parquet``."""
        from .metrics import summarize_groups
        from .utils.trajectory_logging import write_trajectory_groups_parquet

        if step is None:
            step = await self.get_step() if self.trainable else 0
        out_dir = self._get_output_dir()
        os.makedirs(out_dir, exist_ok=True)
        row: dict[str, Any] = {"step": step, "recorded_at": time.time()}
        if trajectories is not None:
            groups = [g if isinstance(g, TrajectoryGroup) else TrajectoryGroup([g]) for g in trajectories]
            write_trajectory_groups_parquet(groups, f"{out_dir}/trajectories/{split}/{step:04d}.parquet")
            for k, v in summarize_groups(groups).items():
                row[f"{split}/{k}"] = v
        for k, v in (metrics or {}).items():
            key = k if "/" in k else f"{split}/{k}"
            row[key] = v
        with open(f"{out_dir}/history.jsonl", "a") as f:
            f.write(json.dumps(row) + "\n")

    async def get_step(self) -> int:
        if self.trainable:
            return await self.backend()._get_step(self)  # type: ignore[attr-defined]
        return 0


class TrainableModel(Model[ModelConfig, StateType]):
    base_model: str
    lora_config: dict[str, Any] | None = None
    trainable: bool = True

    _internal_config: Any = pydantic.PrivateAttr(default=None)

    def __init__(self, *, _internal_config: dev.InternalModelConfig | None = None, **data: Any) -> None:
        super().__init__(**data)
        if _internal_config is not None:
            self._internal_config = _internal_config

    async def register(self, backend: "Backend", _openai_client_config: dev.OpenAIServerConfig | None = None) -> None:
        await super().register(backend)
        base_url, api_key = await backend._prepare_backend_for_training(self, _openai_client_config)
        self.inference_base_url = base_url
        self.inference_api_key = api_key
        name = getattr(backend, "_model_inference_name", None)
        self.inference_model_name = name(self) if name else self.name

    async def delete_checkpoints(self, best_checkpoint_metric: str = "val/reward") -> None:
        """Keep only the latest checkpoint and the best one by
        ``best_checkpoint_metric`` (mean per step in ``history.jsonl``)."""
        keep = [await self.get_step()]
        hist = os.path.join(self._get_output_dir(), "history.jsonl")
        per_step: dict[int, list[float]] = {}
        if os.path.exists(hist):
            with open(hist) as f:
                for line in f:
                    row = json.loads(line)
                    v = row.get(best_checkpoint_metric)
                    if v is not None:
                        per_step.setdefault(int(row["step"]), []).append(float(v))
        if per_step:
            keep.append(max(per_step, key=lambda s: sum(per_step[s]) / len(per_step[s])))
        await self.backend()._delete_checkpoint_files(self, keep)  # type: ignore[attr-defined]

    async def train_sft(
        self,
        trajectories: Iterable[Trajectory],
        config: TrainSFTConfig | None = None,
        _config: dev.TrainSFTConfig | None = None,
        verbose: bool = False,
    ) -> None:
        metrics_seen = []
        async for m in self.backend()._train_sft(self, trajectories, config or TrainSFTConfig(), _config or {}, verbose):  # type: ignore[attr-defined]
            metrics_seen.append(m)
        if metrics_seen:
            avg = {k: sum(m.get(k, 0.0) for m in metrics_seen) / len(metrics_seen) for k in metrics_seen[-1]}
            await self.log(metrics=avg, split="train")


def _deep_merge(a: dict[str, Any], b: dict[str, Any]) -> dict[str, Any]:
    out = dict(a)
    for k, v in b.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = _deep_merge(out[k], v)
        else:
            out[k] = v
    return out

"""``ServerlessBackend``: training on the hosted W&B training service.

Role of the reference ``src/art/serverless/backend.py`` and ``client.py``:
the model lives on the service; ``train`` uploads the trajectory groups as a
training job with the experimental training config, then follows the job's
event stream (``training_started`` -> ``gradient_step``* -> ``training_ended`` /
``training_failed``) and yields the gradient-step metrics.  Inference goes to
the service's OpenAI-compatible endpoint with the same API key.

The REST surface (paths, bodies, cursor pages ``{"data": [...], "has_more"}``
with ``after`` = the last item's id) is the service's and is kept as it is;
the client is this package's own small async client over ``httpx`` with
bounded retries on 408 / 409 / 429 / 5xx and connection errors.  Artifact
transfers that go through the ``wandb`` SDK (checkpoint pulls, forks) need
that SDK, which this image does not have: those methods raise.
"""

from __future__ import annotations

import asyncio
import os
from dataclasses import dataclass
from typing import Any, AsyncIterator, Iterable

from ..trajectories import TrajectoryGroup

DEFAULT_BASE_URL = "https://api.training.wandb.ai/v1"
_RETRY_STATUS = {408, 409, 429, 500, 502, 503, 504}

# experimental training config fields the service accepts
EXPERIMENTAL_KEYS = (
    "advantage_balance", "allow_training_without_logprobs", "epsilon", "epsilon_high",
    "importance_sampling_level", "kimi_k2_tau", "kl_penalty_coef", "kl_penalty_reference_step",
    "kl_penalty_source", "kl_penalty_step_lag", "kl_ref_adapter_path", "learning_rate",
    "logprob_calculation_chunk_size", "loss_fn", "mask_prob_ratio",
    "max_negative_advantage_importance_sampling_weight", "normalize_advantages",
    "num_trajectories_learning_rate_multiplier_power", "packed_sequence_length", "plot_tensors", "ppo",
    "precalculate_logprobs", "scale_learning_rate_by_reward_std_dev", "scale_rewards",
    "truncated_importance_sampling",
)


class ServerlessAPIError(RuntimeError):
    def __init__(self, status: int, body: str) -> None:
        super().__init__(f"training service returned {status}: {body[:500]}")
        self.status = status


@dataclass
class RemoteModel:
    id: str
    entity: str
    project: str
    name: str
    base_model: str
    run_id: str | None = None


class ServerlessClient:
    """Async REST client of the training service."""

    def __init__(self, api_key: str | None = None, base_url: str | None = None, *, max_retries: int = 3,
                 timeout_s: float = 600.0, transport: Any = None) -> None:
        import httpx

        self.api_key = api_key or os.environ.get("WANDB_API_KEY")
        if not self.api_key:
            raise ValueError("the training service needs an API key (api_key= or WANDB_API_KEY)")
        self.base_url = (base_url or os.environ.get("WANDB_BASE_URL_TRAINING") or DEFAULT_BASE_URL).rstrip("/")
        self.max_retries = max_retries
        self._http = httpx.AsyncClient(base_url=self.base_url, timeout=timeout_s, transport=transport,
                                       headers={"Authorization": f"Bearer {self.api_key}"})

    async def close(self) -> None:
        await self._http.aclose()

    async def request(self, method: str, path: str, *, json: Any = None, params: dict | None = None) -> Any:
        import httpx

        delay = 0.5
        for attempt in range(self.max_retries + 1):
            try:
                r = await self._http.request(method, path, json=json,
                                             params={k: v for k, v in (params or {}).items() if v is not None})
            except (httpx.ConnectError, httpx.ReadTimeout, httpx.RemoteProtocolError):
                if attempt == self.max_retries:
                    raise
                await asyncio.sleep(delay)
                delay *= 2
                continue
            if r.status_code in _RETRY_STATUS and attempt < self.max_retries:
                await asyncio.sleep(delay)
                delay *= 2
                continue
            if r.status_code >= 400:
                raise ServerlessAPIError(r.status_code, r.text)
            return r.json() if r.content else None
        raise RuntimeError("unreachable")

    async def pages(self, path: str, **params: Any) -> AsyncIterator[dict]:
        """Items of a cursor-paginated list (``after`` = the last item's id)."""
        after = params.pop("after", None)
        while True:
            page = await self.request("GET", path, params={**params, "after": after})
            items = page.get("data", [])
            for it in items:
                yield it
            if not page.get("has_more") or not items:
                return
            after = items[-1]["id"]

    # ------------------------------------------------------------------ resources
    async def create_model(self, *, entity: str | None, project: str, name: str, base_model: str,
                           return_existing: bool = True) -> RemoteModel:
        d = await self.request("POST", "/preview/models", json={
            "entity": entity, "project": project, "name": name, "base_model": base_model,
            "return_existing": return_existing})
        return RemoteModel(**{k: d.get(k) for k in ("id", "entity", "project", "name", "base_model", "run_id")})

    async def log(self, model_id: str, trajectory_groups: list[TrajectoryGroup], split: str) -> None:
        await self.request("POST", f"/preview/models/{model_id}/log", json={
            "trajectory_groups": [g.model_dump(mode="json") for g in trajectory_groups], "split": split})

    async def delete_model(self, model_id: str) -> None:
        await self.request("DELETE", f"/preview/models/{model_id}")

    def checkpoints(self, model_id: str, *, order: str = "desc", limit: int | None = None) -> AsyncIterator[dict]:
        return self.pages(f"/preview/models/{model_id}/checkpoints", order=order, limit=limit)

    async def delete_checkpoints(self, model_id: str, steps: list[int]) -> dict:
        return await self.request("DELETE", f"/preview/models/{model_id}/checkpoints", json={"steps": steps})

    async def create_training_job(self, model_id: str, trajectory_groups: list[TrajectoryGroup],
                                  experimental_config: dict) -> str:
        d = await self.request("POST", "/preview/training-jobs", json={
            "model_id": model_id, "trajectory_groups": [g.model_dump(mode="json") for g in trajectory_groups],
            "experimental_config": experimental_config})
        return d["id"]

    async def create_sft_job(self, model_id: str, training_data_url: str, config: dict) -> str:
        d = await self.request("POST", "/preview/sft-training-jobs", json={
            "model_id": model_id, "training_data_url": training_data_url, "config": config})
        return d["id"]

    def job_events(self, job_id: str, *, after: str | None = None, sft: bool = False) -> AsyncIterator[dict]:
        kind = "sft-training-jobs" if sft else "training-jobs"
        return self.pages(f"/preview/{kind}/{job_id}/events", after=after)


class ServerlessBackend:
    """Backend whose models train on the hosted service (the ``Backend``
    protocol of ``backend.py``: register, train, get_step, delete, log)."""

    def __init__(self, *, api_key: str | None = None, base_url: str | None = None, poll_interval_s: float = 1.0,
                 transport: Any = None) -> None:
        self._client = ServerlessClient(api_key, base_url, transport=transport)
        self._poll = poll_interval_s

    async def close(self) -> None:
        await self._client.close()

    async def __aenter__(self) -> "ServerlessBackend":
        return self

    async def __aexit__(self, *exc: Any) -> None:
        await self.close()

    async def register(self, model: Any) -> None:
        remote = await self._client.create_model(
            entity=getattr(model, "entity", None), project=model.project, name=model.name,
            base_model=model.base_model)
        model.id = remote.id
        model.entity = remote.entity
        model.run_id = remote.run_id

    async def delete(self, model: Any) -> None:
        await self._client.delete_model(model.id)

    async def _get_step(self, model: Any) -> int:
        async for ck in self._client.checkpoints(model.id, order="desc", limit=1):
            return int(ck["step"])
        return 0

    async def _delete_checkpoint_files(self, model: Any, steps_to_keep: list[int]) -> None:
        keep = set(steps_to_keep)
        drop = [int(ck["step"]) async for ck in self._client.checkpoints(model.id) if int(ck["step"]) not in keep]
        if drop:
            await self._client.delete_checkpoints(model.id, drop)

    async def _log(self, model: Any, trajectory_groups: list[TrajectoryGroup], split: str = "val") -> None:
        await self._client.log(model.id, trajectory_groups, split)

    async def _prepare_backend_for_training(self, model: Any, config: Any = None) -> tuple[str, str]:
        return self._client.base_url, self._client.api_key

    async def train(self, model: Any, trajectory_groups: Iterable[TrajectoryGroup], *, learning_rate: float = 5e-6,
                    loss_fn: str = "cispo", **kwargs: Any) -> dict[str, float]:
        """Run one training job; returns the metrics of its last gradient step
        (the per-step metrics stream through :meth:`train_iter`)."""
        last: dict[str, float] = {}
        async for m in self.train_iter(model, trajectory_groups, learning_rate=learning_rate, loss_fn=loss_fn,
                                       **kwargs):
            last = m
        return last

    async def train_iter(self, model: Any, trajectory_groups: Iterable[TrajectoryGroup], *,
                         learning_rate: float = 5e-6, loss_fn: str = "cispo", **kwargs: Any
                         ) -> AsyncIterator[dict[str, float]]:
        groups = list(trajectory_groups)
        unknown = set(kwargs) - set(EXPERIMENTAL_KEYS)
        if unknown:
            raise ValueError(f"not accepted by the training service: {sorted(unknown)}")
        cfg = {k: kwargs.get(k) for k in EXPERIMENTAL_KEYS}
        cfg.update(learning_rate=learning_rate, loss_fn=loss_fn, ppo=loss_fn == "ppo")
        job = await self._client.create_training_job(model.id, groups, cfg)
        after = None
        steps = None
        while True:
            await asyncio.sleep(self._poll)
            async for ev in self._client.job_events(job, after=after):
                after = ev["id"]
                kind, data = ev["type"], ev.get("data") or {}
                if kind == "training_started":
                    steps = data.get("num_sequences")
                elif kind == "gradient_step":
                    out = {k: float(v) for k, v in data.items() if isinstance(v, (int, float))}
                    if steps is not None:
                        out["data/step_num_gradient_steps"] = float(steps)
                    yield out
                elif kind == "training_ended":
                    return
                elif kind == "training_failed":
                    raise RuntimeError(f"training job failed: {data.get('error_message', 'unknown error')}")

    async def _experimental_pull_model_checkpoint(self, *args: Any, **kwargs: Any) -> str:
        raise NotImplementedError("checkpoint artifacts are fetched through the wandb SDK, not installed here")

    async def _experimental_fork_checkpoint(self, *args: Any, **kwargs: Any) -> int:
        raise NotImplementedError("forks copy wandb artifacts through the wandb SDK, not installed here")

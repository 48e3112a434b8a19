"""HTTP client of a tau-bench environment server.

Wire format shared with the reference's ``src/art/tau_bench/client.py`` (the
server is the same): ``GET /scenarios?domain=&split=`` ->
``{"scenarios": [{"domain", "task"}]}``; ``POST /environments`` with
``domain``, ``task_id`` and optional user-simulator / retrieval settings ->
``{"id", "observation", "info"}``; ``POST /environments/{id}/step`` with
``{"action"}`` -> adds ``reward``, ``terminated``, ``truncated``;
``DELETE /environments/{id}`` -> ``{"id", "deleted"}``.  Bearer auth from
``TAU_BENCH_API_KEY``; base URL from ``TAU_BENCH_BASE_URL``.  5xx / 429
answers and transport errors are retried with capped exponential backoff.
"""

from __future__ import annotations

import asyncio
import os
import uuid
from contextlib import asynccontextmanager
from typing import Any, AsyncIterator

import httpx
from pydantic import BaseModel

Json = dict[str, Any]


class Task(BaseModel):
    id: str
    description: Json | str | None = None
    user_scenario: Json | str | None = None
    ticket: str | None = None
    initial_state: Json | None = None
    evaluation_criteria: Json | None = None
    issues: list[Json | str] | None = None
    required_documents: list[str] | None = None
    user_tools: list[str] | None = None


class Scenario(BaseModel):
    domain: str
    task: Task


class EnvironmentResponse(BaseModel):
    id: str
    observation: str
    info: dict[str, Any]


class StepEnvironmentResponse(EnvironmentResponse):
    reward: float
    terminated: bool
    truncated: bool


class DeleteEnvironmentResponse(BaseModel):
    id: str
    deleted: bool


def _drop_none(d: dict[str, Any]) -> dict[str, Any]:
    return {k: v for k, v in d.items() if v is not None}


class TauBenchClient:
    def __init__(self, *, base_url: str | None = None, api_key: str | None = None, timeout: float | None = 300.0,
                 http_client: httpx.AsyncClient | None = None, status_retries: int = 3,
                 retry_base_delay: float = 0.5, retry_max_delay: float = 8.0) -> None:
        self.api_key = api_key if api_key is not None else os.getenv("TAU_BENCH_API_KEY")
        self.status_retries = status_retries
        self.retry_base_delay, self.retry_max_delay = retry_base_delay, retry_max_delay
        self._owns = http_client is None
        self._client = http_client or httpx.AsyncClient(
            base_url=base_url or os.getenv("TAU_BENCH_BASE_URL") or "http://localhost:8000", timeout=timeout)

    async def close(self) -> None:
        if self._owns:
            await self._client.aclose()

    async def __aenter__(self) -> "TauBenchClient":
        return self

    async def __aexit__(self, *exc: object) -> None:
        await self.close()

    async def _request(self, method: str, url: str, **kw: Any) -> Any:
        headers = {"X-Request-ID": str(uuid.uuid4())}
        if self.api_key:
            headers["Authorization"] = f"Bearer {self.api_key}"
        delay = self.retry_base_delay
        for attempt in range(self.status_retries + 1):
            last = attempt == self.status_retries
            try:
                r = await self._client.request(method, url, headers=headers, **kw)
            except httpx.TransportError:
                if last:
                    raise
            else:
                if r.status_code < 500 and r.status_code != 429:
                    if r.status_code >= 400:
                        try:
                            detail = r.json().get("detail")
                        except ValueError:
                            detail = r.text
                        raise httpx.HTTPStatusError(f"{method} {url}: {r.status_code} {detail}", request=r.request,
                                                    response=r)
                    return r.json()
                if last:
                    r.raise_for_status()
            await asyncio.sleep(delay)
            delay = min(delay * 2, self.retry_max_delay)
        raise AssertionError("unreachable")

    async def get_scenarios(self, *, domain: str | None = None, split: str | None = None) -> list[Scenario]:
        data = await self._request("GET", "/scenarios", params=_drop_none({"domain": domain, "split": split}))
        return [Scenario.model_validate(s) for s in data["scenarios"]]

    async def create_environment(self, *, domain: str, task_id: str, user_llm: str | None = None,
                                 user_llm_args: dict[str, Any] | None = None, retrieval_config: str | None = None,
                                 retrieval_config_kwargs: dict[str, Any] | None = None,
                                 idle_timeout_seconds: float | None = None) -> EnvironmentResponse:
        body = _drop_none({"domain": domain, "task_id": task_id, "user_llm": user_llm, "user_llm_args": user_llm_args,
                           "retrieval_config": retrieval_config, "retrieval_config_kwargs": retrieval_config_kwargs,
                           "idle_timeout_seconds": idle_timeout_seconds})
        return EnvironmentResponse.model_validate(await self._request("POST", "/environments", json=body))

    async def step_environment(self, env_id: str, action: str) -> StepEnvironmentResponse:
        data = await self._request("POST", f"/environments/{env_id}/step", json={"action": action})
        return StepEnvironmentResponse.model_validate(data)

    async def delete_environment(self, env_id: str) -> DeleteEnvironmentResponse:
        return DeleteEnvironmentResponse.model_validate(await self._request("DELETE", f"/environments/{env_id}"))

    @asynccontextmanager
    async def environment(self, **kw: Any) -> AsyncIterator[EnvironmentResponse]:
        env = await self.create_environment(**kw)
        try:
            yield env
        finally:
            await self.delete_environment(env.id)


_default: TauBenchClient | None = None


def default_client() -> TauBenchClient:
    global _default
    if _default is None:
        _default = TauBenchClient()
    return _default


async def get_scenarios(*, domain: str | None = None, split: str | None = None,
                        client: TauBenchClient | None = None) -> list[Scenario]:
    return await (client or default_client()).get_scenarios(domain=domain, split=split)

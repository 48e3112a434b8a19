"""``RemoteBackend``: the Backend protocol over HTTP to a ``art-b200 run``
server (``cli.py``), so a notebook or a CPU-only machine drives training on
a GPU host.  Same role as the reference's client for ``art run``
(``src/art/cli.py:229``).  Models and trajectory groups travel as their
pydantic JSON; the server rebuilds them and calls its ``LocalBackend``."""

from __future__ import annotations

from typing import Any, AsyncIterator, Iterable

from ..trajectories import Trajectory, TrajectoryGroup
from ..types import LocalTrainResult, TrainSFTConfig


def _model_json(model: Any) -> dict[str, Any]:
    d = model.model_dump(mode="json")
    internal = getattr(model, "_internal_config", None)
    if internal:
        d["_internal_config"] = dict(internal)
    return d


class RemoteBackend:
    def __init__(self, base_url: str = "http://127.0.0.1:7999", timeout_s: float = 3600.0) -> None:
        import httpx

        self.base_url = base_url.rstrip("/")
        self._client = httpx.AsyncClient(base_url=self.base_url, timeout=timeout_s)
        self._steps: dict[str, int] = {}

    async def _post(self, path: str, body: dict[str, Any]) -> Any:
        r = await self._client.post(path, json=body)
        if r.status_code >= 400:
            raise RuntimeError(f"{path}: HTTP {r.status_code}: {r.text[:2000]}")
        return r.json()

    async def healthcheck(self) -> bool:
        r = await self._client.get("/healthcheck")
        return r.status_code == 200

    async def register(self, model: Any) -> None:
        await self._post("/register", {"model": _model_json(model)})

    async def _get_step(self, model: Any) -> int:
        step = int(await self._post("/_get_step", {"model": _model_json(model)}))
        self._steps[model.name] = step
        return step

    def _model_inference_name(self, model: Any, step: int | None = None) -> str:
        s = step if step is not None else self._steps.get(model.name)
        return f"{model.name}@{s}" if s is not None else model.name

    async def _prepare_backend_for_training(self, model: Any, config: dict | None = None) -> tuple[str, str]:
        url, key = await self._post("/_prepare_backend_for_training", {"model": _model_json(model), "config": config})
        await self._get_step(model)
        return url, key

    async def _delete_checkpoint_files(self, model: Any, steps_to_keep: list[int]) -> None:
        await self._post("/_delete_checkpoint_files", {"model": _model_json(model), "steps_to_keep": steps_to_keep})

    async def train(self, model: Any, trajectory_groups: Iterable[TrajectoryGroup], **kwargs: Any) -> LocalTrainResult:
        groups = [g.model_dump(mode="json") for g in trajectory_groups]
        out = await self._post("/train", {"model": _model_json(model), "trajectory_groups": groups, "kwargs": kwargs})
        self._steps[model.name] = int(out["step"])
        return LocalTrainResult(step=int(out["step"]), metrics=out["metrics"], checkpoint_path=out["checkpoint_path"])

    async def _train_sft(self, model: Any, trajectories: Iterable[Trajectory], config: TrainSFTConfig,
                         dev_config: dict, verbose: bool = False) -> AsyncIterator[dict[str, float]]:
        rows = await self._post("/_train_sft", {
            "model": _model_json(model), "trajectories": [t.model_dump(mode="json") for t in trajectories],
            "config": config.model_dump(mode="json"),
        })
        for r in rows:
            yield r

    async def close(self) -> None:
        try:
            await self._post("/close", {})
        finally:
            await self._client.aclose()

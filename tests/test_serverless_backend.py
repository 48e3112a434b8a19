"""ServerlessBackend against a fake training service (httpx mock transport):
model registration, a training job followed through its event pages,
checkpoint listing / pruning with cursor pages, retries and auth."""

import asyncio
import json

import httpx
import pytest

from art_mlx_b200.backends.serverless import ServerlessBackend
from art_mlx_b200.trajectories import Trajectory, TrajectoryGroup


class FakeService:
    def __init__(self):
        self.calls = []
        self.jobs = {}
        self.checkpoints = [{"id": f"ck{s}", "step": s, "metrics": {}} for s in (3, 2, 1)]
        self.fail_once = {"/preview/training-jobs"}

    def __call__(self, request: httpx.Request) -> httpx.Response:
        assert request.headers["authorization"] == "Bearer k"
        path, method = request.url.path.removeprefix("/v1"), request.method
        self.calls.append((method, path))
        body = json.loads(request.content) if request.content else None
        if path in self.fail_once:  # a transient error the client retries
            self.fail_once.discard(path)
            return httpx.Response(429, json={"error": "slow down"})
        if method == "POST" and path == "/preview/models":
            return httpx.Response(200, json={"id": "m1", "entity": "e", "project": body["project"],
                                             "name": body["name"], "base_model": body["base_model"], "run_id": "r"})
        if method == "GET" and path == "/preview/models/m1/checkpoints":
            after = request.url.params.get("after")
            items = self.checkpoints
            if after:
                i = [c["id"] for c in items].index(after)
                items = items[i + 1 :]
            limit = int(request.url.params.get("limit", 2))
            return httpx.Response(200, json={"data": items[:limit], "has_more": len(items) > limit})
        if method == "DELETE" and path == "/preview/models/m1/checkpoints":
            self.checkpoints = [c for c in self.checkpoints if c["step"] not in body["steps"]]
            return httpx.Response(200, json={"deleted_count": len(body["steps"]), "not_found_steps": []})
        if method == "POST" and path == "/preview/training-jobs":
            assert len(body["trajectory_groups"]) == 1 and body["experimental_config"]["learning_rate"] == 1e-5
            self.jobs["j1"] = [
                {"id": "e1", "type": "training_started", "data": {"num_sequences": 2}},
                {"id": "e2", "type": "gradient_step", "data": {"loss": 0.5}},
                {"id": "e3", "type": "gradient_step", "data": {"loss": 0.25}},
                {"id": "e4", "type": "training_ended", "data": {}},
            ]
            return httpx.Response(200, json={"id": "j1"})
        if method == "GET" and path == "/preview/training-jobs/j1/events":
            ev = self.jobs["j1"]
            after = request.url.params.get("after")
            if after:
                ev = ev[[e["id"] for e in ev].index(after) + 1 :]
            return httpx.Response(200, json={"data": ev[:2], "has_more": len(ev) > 2})
        return httpx.Response(404, json={"error": path})


class M:
    name, project, base_model = "agent", "proj", "Qwen/Qwen3-8B"


def test_serverless_backend_flow():
    svc = FakeService()

    async def go():
        b = ServerlessBackend(api_key="k", base_url="https://svc/v1", poll_interval_s=0.0,
                              transport=httpx.MockTransport(svc))
        m = M()
        await b.register(m)
        assert m.id == "m1"
        assert await b._get_step(m) == 3
        g = TrajectoryGroup([Trajectory(messages_and_choices=[{"role": "user", "content": "x"}], reward=1.0)])
        steps = [x async for x in b.train_iter(m, [g], learning_rate=1e-5)]
        assert [s["loss"] for s in steps] == [0.5, 0.25] and steps[0]["data/step_num_gradient_steps"] == 2.0
        await b._delete_checkpoint_files(m, [3])
        assert [c["step"] for c in svc.checkpoints] == [3]
        with pytest.raises(ValueError):
            await b.train(m, [g], not_a_knob=1)
        await b.close()

    asyncio.run(go())
    assert ("POST", "/preview/training-jobs") in svc.calls and svc.calls.count(("POST", "/preview/training-jobs")) == 2

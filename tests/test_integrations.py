"""tau-bench client + rollout against a fake environment server (httpx
MockTransport), and guided-completion parameters for distillation."""

import asyncio
import json
import httpx

from art_mlx_b200.guided_completion import freeze_tool_schema, get_guided_completion_params
from art_mlx_b200.tau_bench import Scenario, TauBenchClient, rollout, tool_call_action

TOOLS = [{"type": "function", "function": {"name": "get_order", "parameters": {
    "type": "object", "properties": {"order_id": {"type": "string"}, "n": {"type": "integer"}}}}}]


def _fake_server():
    envs, log = {}, []
    flaky = {"left": 1}

    def handler(request: httpx.Request) -> httpx.Response:
        log.append((request.method, request.url.path, request.headers.get("authorization")))
        if request.url.path == "/scenarios":
            if flaky["left"]:
                flaky["left"] -= 1
                return httpx.Response(503)  # retried by the client
            return httpx.Response(200, json={"scenarios": [{"domain": "retail", "task": {"id": "t1"}}]})
        if request.url.path == "/environments" and request.method == "POST":
            body = json.loads(request.content)
            envs["e1"] = {"task": body["task_id"], "steps": 0}
            return httpx.Response(200, json={"id": "e1", "observation": "user: where is my order?",
                                             "info": {"policy": "be helpful", "tools": TOOLS}})
        if request.url.path == "/environments/e1/step":
            action = json.loads(request.content)["action"]
            envs["e1"]["steps"] += 1
            envs["e1"].setdefault("actions", []).append(action)
            if action.startswith("get_order("):
                return httpx.Response(200, json={"id": "e1", "observation": "tool: shipped", "info": {},
                                                 "reward": 0.0, "terminated": False, "truncated": False})
            return httpx.Response(200, json={"id": "e1", "observation": "user: thanks", "info": {"user_message_cost": 0.01},
                                             "reward": 1.0, "terminated": True, "truncated": False})
        if request.url.path == "/environments/e1" and request.method == "DELETE":
            envs["e1"]["deleted"] = True
            return httpx.Response(200, json={"id": "e1", "deleted": True})
        return httpx.Response(404, json={"detail": "no route"})

    return handler, envs, log


class _Policy:
    """OpenAI-like client: first a tool call, then a text answer."""

    def __init__(self):
        self.calls = 0
        from types import SimpleNamespace

        self.chat = SimpleNamespace(completions=SimpleNamespace(create=self.create))

    async def create(self, **kw):
        from openai.types.chat import ChatCompletion

        self.calls += 1
        if self.calls == 1:
            msg = {"role": "assistant", "content": None, "tool_calls": [
                {"id": "c1", "type": "function", "function": {"name": "get_order",
                                                              "arguments": '{"order_id": "A7", "n": 2}'}}]}
        else:
            msg = {"role": "assistant", "content": "It has shipped."}
        return ChatCompletion.model_validate({
            "id": "x", "object": "chat.completion", "created": 0, "model": "m",
            "choices": [{"index": 0, "finish_reason": "stop", "message": msg}],
            "usage": {"prompt_tokens": 90, "completion_tokens": 10, "total_tokens": 100}})


def test_tau_bench_client_and_rollout():
    handler, envs, log = _fake_server()

    async def go():
        http = httpx.AsyncClient(transport=httpx.MockTransport(handler), base_url="http://tau")
        client = TauBenchClient(http_client=http, api_key="k", retry_base_delay=0.001)
        scen = await client.get_scenarios(domain="retail")
        assert isinstance(scen[0], Scenario) and scen[0].task.id == "t1"
        traj = await rollout(scen[0], _Policy(), model_name="m", client=client, max_turns=5)
        await http.aclose()
        return traj

    traj = asyncio.run(go())
    assert traj.reward == 1.0 and traj.metrics["num_turns"] == 2 and abs(traj.metrics["cost/user"] - 0.01) < 1e-12
    assert envs["e1"]["actions"][0] == "get_order(order_id='A7', n=2)"
    assert envs["e1"]["deleted"] is True
    assert all(a == "Bearer k" for _, _, a in log)
    assert traj.messages_and_choices[0]["content"] == "be helpful"
    assert traj.messages_and_choices[1]["content"] == "where is my order?"


def test_guided_completion_params():
    call = {"id": "c", "type": "function", "function": {"name": "get_order", "arguments": '{"order_id": "A7"}'}}
    comp = {"choices": [{"message": {"role": "assistant", "content": None, "tool_calls": [call]}}]}
    choice, tool_choice, tools = get_guided_completion_params(comp, TOOLS)
    assert choice is None and tool_choice == {"type": "function", "function": {"name": "get_order"}}
    params = tools[0]["function"]["parameters"]
    assert params["properties"]["order_id"]["enum"] == ["A7"] and params["required"] == ["order_id"]
    assert TOOLS[0]["function"]["parameters"]["properties"]["order_id"] == {"type": "string"}  # not mutated
    text = {"choices": [{"message": {"role": "assistant", "content": "hello"}}]}
    assert get_guided_completion_params(text) == (["hello"], None, None)
    assert freeze_tool_schema(TOOLS[0], {})["function"]["parameters"]["properties"] == {}
    assert tool_call_action(call) == "get_order(order_id='A7')"

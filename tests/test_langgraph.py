"""LangGraph-style rollouts: chat-model calls made through ``init_chat_model``
inside ``wrap_rollout`` become the trajectory's histories (reference
counterpart: ``src/art/langgraph/llm_wrapper.py``).  LangChain is not needed:
the fakes below speak its message protocol."""

import asyncio
import dataclasses
from typing import Any

import pydantic
import pytest

from art_mlx_b200 import langgraph as lg
from art_mlx_b200.trajectories import Trajectory


@dataclasses.dataclass
class Msg:
    type: str
    content: str
    tool_calls: list | None = None
    tool_call_id: str | None = None
    response_metadata: dict | None = dataclasses.field(default=None, compare=False)


def _ai(content, tool_calls=None):
    lp = {"content": [{"token": "x", "logprob": -0.5, "bytes": None, "top_logprobs": []}]}
    return Msg("ai", content, tool_calls, response_metadata={"logprobs": lp, "finish_reason": "stop"})


class FakeChat:
    """Replies from a script; records what it was asked."""

    def __init__(self, replies, delay: float = 0.0):
        self.replies, self.delay, self.seen, self.tools = list(replies), delay, [], None

    def invoke(self, input, config=None, **kw):
        self.seen.append(input)
        return self.replies.pop(0)

    async def ainvoke(self, input, config=None, **kw):
        await asyncio.sleep(self.delay)
        return self.invoke(input, config)

    def bind_tools(self, tools, **kw):
        self.tools = tools
        return self


class FakeModel:
    inference_base_url, inference_api_key, inference_model_name = "http://127.0.0.1:1/v1", "k", "m@3"


def test_calls_fold_into_main_and_additional_histories(tmp_path):
    sys_, h1 = Msg("system", "be brief"), Msg("human", "2+2?")
    a1 = _ai("", tool_calls=[{"name": "add", "args": '{"a": 2, "b": 2}', "id": "c1"}])
    a2, a3 = _ai("4"), _ai("summary")
    tool = Msg("tool", "4", tool_call_id="c1")
    chat = FakeChat([a1, a2, a3])

    async def rollout():
        llm = lg.init_chat_model(chat).bind_tools([{"name": "add", "parameters": {"type": "object"}}])
        out = await llm.ainvoke([sys_, h1])
        assert out.tool_calls[0]["args"] == {"a": 2, "b": 2}  # decoded from the JSON string
        await llm.ainvoke([sys_, h1, out, tool])  # continues the first conversation
        await llm.ainvoke([Msg("system", "summarise"), Msg("human", "the chat")])  # a second one
        return Trajectory(reward=1.0)

    t = asyncio.run(lg.wrap_rollout(FakeModel(), rollout, log_dir=str(tmp_path))())
    roles = [m["role"] if isinstance(m, dict) else "choice" for m in t.messages_and_choices]
    assert roles == ["system", "user", "choice", "tool", "choice"]
    first = t.messages_and_choices[2]
    assert first.message.tool_calls[0].function.name == "add"
    assert first.message.tool_calls[0].function.arguments == '{"a": 2, "b": 2}'
    assert t.tools == [{"type": "function", "function": {"name": "add", "parameters": {"type": "object"}}}]
    assert len(t.additional_histories) == 1
    assert [type(m).__name__ if not isinstance(m, dict) else m["role"]
            for m in t.additional_histories[0].messages_and_choices] == ["system", "user", "Choice"]
    assert t.reward == 1.0 and t.messages()[-1]["content"] == "4"
    assert len(list(tmp_path.iterdir())) == 1  # the readable call log


def test_a_new_human_turn_continues_the_thread():
    sys_, h1, h2 = Msg("system", "s"), Msg("human", "hi"), Msg("human", "more")
    a1, a2 = _ai("hello"), _ai("sure")
    chat = FakeChat([a1, a2])

    async def rollout():
        llm = lg.init_chat_model(chat)
        r = await llm.ainvoke([sys_, h1])
        await llm.ainvoke([sys_, h1, r, h2])
        return Trajectory()

    t = asyncio.run(lg.wrap_rollout(FakeModel(), rollout, log_dir=None)())
    assert len(t.additional_histories) == 0
    assert [m["content"] if isinstance(m, dict) else m.message.content for m in t.messages_and_choices] == [
        "s", "hi", "hello", "more", "sure"]


def test_concurrent_rollouts_keep_their_own_calls():
    async def rollout(i):
        llm = lg.init_chat_model(FakeChat([_ai(f"a{i}")], delay=0.01 * (3 - i)))
        await llm.ainvoke([Msg("human", f"q{i}")])
        return Trajectory()

    async def main():
        w = lg.wrap_rollout(FakeModel(), rollout, log_dir=None)
        return await asyncio.gather(*(w(i) for i in range(3)))

    for i, t in enumerate(asyncio.run(main())):
        assert t.messages_and_choices[0]["content"] == f"q{i}"
        assert t.messages_and_choices[1].message.content == f"a{i}"


class Answer(pydantic.BaseModel):
    """The final answer."""

    value: int


def test_structured_output_and_sync_invoke():
    chat = FakeChat([_ai("", tool_calls=[{"name": "Answer", "args": {"value": 7}, "id": "c"}])])

    async def rollout():
        ans = lg.init_chat_model(chat).with_structured_output(Answer).invoke([Msg("human", "?")])
        assert ans == Answer(value=7)
        return Trajectory()

    t = asyncio.run(lg.wrap_rollout(FakeModel(), rollout, log_dir=None)())
    assert chat.tools == [Answer]
    assert t.tools[0]["function"]["name"] == "Answer"
    assert t.tools[0]["function"]["parameters"]["properties"]["value"]["type"] == "integer"


def test_invoke_timeout_bounds_a_slow_call():
    async def rollout():
        llm = lg.init_chat_model(FakeChat([_ai("late")], delay=1.0), invoke_timeout=0.05)
        await llm.ainvoke([Msg("human", "?")])
        return Trajectory()

    with pytest.raises(asyncio.TimeoutError):
        asyncio.run(lg.wrap_rollout(FakeModel(), rollout, log_dir=None)())


def test_init_chat_model_arguments():
    lg.start_rollout("http://127.0.0.1:1/v1", "k", "m", log_dir=None)
    with pytest.raises(ValueError):
        lg.init_chat_model("m", model_provider="anthropic")
    with pytest.raises(ValueError):
        lg.init_chat_model(configurable_fields=("model",))  # type: ignore[arg-type]
    assert isinstance(lg.init_chat_model(FakeChat([])), lg.LoggingChatModel)


def test_with_config_repoints_at_the_current_rollout():
    built: list[dict[str, Any]] = []

    def factory(ep):
        built.append(ep)
        return FakeChat([_ai("x")])

    lg.start_rollout("http://a/v1", "k", "m@1", log_dir=None)
    llm = lg.LoggingChatModel(factory(lg.current_recorder().endpoint), factory=factory)
    lg.start_rollout("http://b/v1", "k", "m@2", log_dir=None)
    llm.with_config({"tags": ["t"]})
    assert built[-1]["base_url"] == "http://b/v1" and built[-1]["model"] == "m@2"
    assert llm.invoke([Msg("human", "q")]).content == "x"
    assert len(lg.current_recorder().calls) == 1


def test_message_conversion_rejects_unknown_objects():
    with pytest.raises(TypeError):
        lg.message_to_openai(object())
    assert lg.message_to_openai(Msg("tool", "r", tool_call_id="c")) == {"role": "tool", "content": "r",
                                                                       "tool_call_id": "c"}

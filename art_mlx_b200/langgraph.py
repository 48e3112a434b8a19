"""LangGraph / LangChain rollouts that become trajectories.

Role of the reference's ``src/art/langgraph/llm_wrapper.py:100-295`` and
``message_utils.py:70-123``: an agent written against LangChain chat models
runs unchanged inside ``wrap_rollout(model, fn)``; every chat-model call made
through ``init_chat_model()`` is recorded, and when the rollout returns its
``Trajectory`` the recorded calls are folded into it as the main history plus
additional histories (one per distinct conversation the agent held).

Own design:

* The record of a rollout is an in-memory ``RolloutRecorder`` held in a
  context variable (so concurrent rollouts in one event loop stay apart); a
  readable text log of the calls is also appended under ``log_dir``.
* LangChain is optional.  Messages are read through LangChain's message
  protocol (``.type`` of ``human``/``ai``/``system``/``tool``/``function``,
  ``.content``, ``.tool_calls``, ``.tool_call_id``, ``.response_metadata``),
  so any chat model that speaks it can be wrapped without importing LangChain;
  only building the default OpenAI-compatible client needs ``langchain_openai``.
* Folding calls into conversations: a call's conversation is its input
  messages followed by its output.  A call whose input, without tool
  messages and without a trailing human turn, equals the non-tool messages of
  a conversation already seen continues that conversation (the longer one
  replaces it); otherwise it starts a new one.  This is the reference's rule,
  kept because agents built on LangGraph re-send the whole history each turn
  and interleave tool results, so prefix identity on the non-tool messages is
  what identifies a thread.
* Assistant outputs carrying ``logprobs`` in their response metadata become
  OpenAI ``Choice`` objects (trainable); the rest become plain message dicts.
"""

from __future__ import annotations

import asyncio
import contextvars
import json
import os
import uuid
from collections.abc import Awaitable, Callable
from typing import Any

from .trajectories import History, Trajectory

DEFAULT_INVOKE_TIMEOUT = 10 * 60
OPENAI_COMPATIBLE_PROVIDERS = {None, "openai", "openai-compatible", "openai_compatible"}

_ROLES = {"human": "user", "ai": "assistant", "system": "system", "tool": "tool", "function": "function",
          "developer": "developer"}
_CLASS_ROLES = {"HumanMessage": "user", "AIMessage": "assistant", "AIMessageChunk": "assistant",
                "SystemMessage": "system", "ToolMessage": "tool", "FunctionMessage": "function"}


class RolloutRecorder:
    """The chat-model calls of one rollout, in the order they completed."""

    def __init__(self, endpoint: dict[str, Any], log_path: str | None = None) -> None:
        self.endpoint = endpoint  # base_url, api_key, model of the rollout's inference server
        self.log_path = log_path
        self.calls: list[dict[str, Any]] = []

    def record(self, call_id: str, input: Any, output: Any, tools: list | None) -> None:
        entry = {"id": call_id, "input": input, "output": output, "tools": tools}
        self.calls.append(entry)
        if self.log_path:
            with open(self.log_path, "a") as f:
                f.write(f"{call_id}: {entry!r}\n")


_CURRENT: contextvars.ContextVar[RolloutRecorder | None] = contextvars.ContextVar("art_langgraph_rollout",
                                                                                  default=None)


def current_recorder() -> RolloutRecorder:
    rec = _CURRENT.get()
    if rec is None:
        raise RuntimeError("no rollout is active: call the chat model inside a function wrapped by wrap_rollout()")
    return rec


def start_rollout(base_url: str | None, api_key: str | None, model: str | None,
                  log_dir: str | None = ".art/langgraph") -> RolloutRecorder:
    """Make a fresh recorder the current one (in this context) and return it."""
    path = None
    if log_dir:
        os.makedirs(log_dir, exist_ok=True)
        path = os.path.join(log_dir, str(uuid.uuid4()))
    rec = RolloutRecorder({"base_url": base_url, "api_key": api_key, "model": model}, path)
    _CURRENT.set(rec)
    return rec


# ---------------------------------------------------------------------------
# messages


def _role(msg: Any) -> str | None:
    t = getattr(msg, "type", None)
    if isinstance(t, str) and t in _ROLES:
        return _ROLES[t]
    return _CLASS_ROLES.get(type(msg).__name__)


def _is_tool_message(msg: Any) -> bool:
    return (msg.get("role") if isinstance(msg, dict) else _role(msg)) == "tool"


def _is_human(msg: Any) -> bool:
    return (msg.get("role") if isinstance(msg, dict) else _role(msg)) == "user"


def message_to_openai(msg: Any) -> dict[str, Any]:
    """A LangChain message (or a dict already in the OpenAI format) as an
    OpenAI chat message dict."""
    if isinstance(msg, dict):
        return msg
    role = _role(msg)
    if role is None:
        raise TypeError(f"unsupported message type: {type(msg).__name__}")
    out: dict[str, Any] = {"role": role, "content": getattr(msg, "content", None) or ""}
    for k in ("tool_calls", "tool_call_id", "function_call"):
        v = getattr(msg, k, None)
        if not v and k == "function_call":
            v = (getattr(msg, "additional_kwargs", None) or {}).get("function_call")
        if v:
            out[k] = v
    return out


def _openai_tool_calls(tool_calls: list[dict[str, Any]]) -> list[dict[str, Any]]:
    """LangChain tool calls ({name, args, id}) in the OpenAI wire format."""
    out = []
    for tc in tool_calls:
        args = tc.get("args", {})
        out.append({"id": tc.get("id") or f"call_{uuid.uuid4().hex[:12]}", "type": "function",
                    "function": {"name": tc["name"],
                                 "arguments": args if isinstance(args, str) else json.dumps(args)}})
    return out


def convert_messages(messages: list[Any]) -> list[Any]:
    """LangChain messages -> the trajectory format.  An assistant message whose
    response metadata holds ``logprobs`` becomes a ``Choice``."""
    from openai.types.chat.chat_completion import Choice
    from openai.types.chat.chat_completion_message import ChatCompletionMessage

    out: list[Any] = []
    for msg in messages:
        meta = getattr(msg, "response_metadata", None) if not isinstance(msg, dict) else None
        if meta and "logprobs" in meta and _role(msg) == "assistant":
            tcs = getattr(msg, "tool_calls", None)
            out.append(Choice(
                index=0,
                finish_reason=meta.get("finish_reason") or ("tool_calls" if tcs else "stop"),
                logprobs=meta.get("logprobs"),
                message=ChatCompletionMessage(role="assistant", content=getattr(msg, "content", None) or None,
                                              tool_calls=_openai_tool_calls(tcs) if tcs else None),
            ))
        else:
            out.append(message_to_openai(msg))
    return out


def _input_messages(input: Any) -> list[Any]:
    if hasattr(input, "to_messages"):  # a ChatPromptValue
        return list(input.to_messages())
    if isinstance(input, str):
        return [{"role": "user", "content": input}]
    return list(input)


def fold_calls(recorder: RolloutRecorder, trajectory: Trajectory) -> Trajectory:
    """Fill ``trajectory`` from the recorded calls: the first conversation is
    its main history, every other one an additional history."""
    convs: list[list[Any]] = []
    tools: list[list | None] = []
    for call in recorder.calls:
        inp = _input_messages(call["input"])
        output = call["output"]
        raw = output.get("raw") if isinstance(output, dict) else output
        conv = inp + [raw]
        key = [m for m in inp if not _is_tool_message(m)]
        if key and _is_human(key[-1]):
            key = key[:-1]
        for i, prev in enumerate(convs):
            if [m for m in prev if not _is_tool_message(m)] == key:
                convs[i], tools[i] = conv, call["tools"]
                break
        else:
            convs.append(conv)
            tools.append(call["tools"])
    for i, conv in enumerate(convs):
        try:
            msgs = convert_messages(conv)
        except (TypeError, ValueError):
            continue  # a conversation the trainer cannot read is left out, as a failed rollout would be
        if i == 0:
            trajectory.messages_and_choices = msgs
            trajectory.tools = tools[i]
        else:
            trajectory.additional_histories.append(History(messages_and_choices=msgs, tools=tools[i]))
    return trajectory


# ---------------------------------------------------------------------------
# tools


def to_openai_tool(tool: Any) -> dict[str, Any]:
    """A tool in the OpenAI ``{"type": "function", "function": {...}}`` form.
    Accepts that form, a bare function spec dict, a pydantic model class, a
    LangChain tool (through LangChain when it is installed) or a plain
    function (name and docstring, arguments unchecked)."""
    if isinstance(tool, dict):
        if tool.get("type") == "function" and "function" in tool:
            return tool
        if "name" in tool:
            return {"type": "function", "function": tool}
    try:
        import pydantic

        if isinstance(tool, type) and issubclass(tool, pydantic.BaseModel):
            return {"type": "function", "function": {"name": tool.__name__, "description": (tool.__doc__ or "").strip(),
                                                     "parameters": tool.model_json_schema()}}
    except ImportError:  # pragma: no cover - pydantic is a dependency
        pass
    try:
        from langchain_core.utils.function_calling import convert_to_openai_tool

        return convert_to_openai_tool(tool)
    except ImportError:
        pass
    if callable(tool):
        return {"type": "function", "function": {"name": getattr(tool, "__name__", "tool"),
                                                 "description": (getattr(tool, "__doc__", "") or "").strip(),
                                                 "parameters": {"type": "object", "properties": {}}}}
    raise TypeError(f"cannot describe {tool!r} as an OpenAI tool")


# ---------------------------------------------------------------------------
# the logged chat model

try:  # behave as a LangChain Runnable when LangChain is there (LangGraph checks for it)
    from langchain_core.runnables import Runnable as _Base
except ImportError:
    _Base = object


class LoggingChatModel(_Base):  # type: ignore[misc,valid-type]
    """Wraps a chat model; every completed call is recorded on the current
    rollout.  Tool-call arguments that arrive as JSON strings are decoded;
    with a structured-output schema the first tool call's arguments are
    validated into it."""

    def __init__(self, llm: Any, *, structured_output: Any = None, tools: list | None = None,
                 invoke_timeout: float | None = DEFAULT_INVOKE_TIMEOUT,
                 factory: Callable[[dict[str, Any]], Any] | None = None) -> None:
        self.llm = llm
        self.structured_output = structured_output
        self.tools = [to_openai_tool(t) for t in tools] if tools else None
        self.invoke_timeout = invoke_timeout
        self.factory = factory

    def _finish(self, input: Any, result: Any) -> Any:
        rec = _CURRENT.get()
        if rec is not None:
            rec.record(str(uuid.uuid4()), input, result, self.tools)
        tcs = getattr(result, "tool_calls", None)
        for tc in tcs or ():
            if isinstance(tc.get("args"), str):
                tc["args"] = json.loads(tc["args"])
        if self.structured_output is not None:
            return self.structured_output.model_validate(tcs[0]["args"] if tcs else None)
        return result

    def invoke(self, input: Any, config: Any = None, **kwargs: Any) -> Any:
        return self._finish(input, self.llm.invoke(input, config=config, **kwargs))

    async def ainvoke(self, input: Any, config: Any = None, **kwargs: Any) -> Any:
        call = self.llm.ainvoke(input, config=config, **kwargs)
        result = await (call if self.invoke_timeout is None else asyncio.wait_for(call, self.invoke_timeout))
        return self._finish(input, result)

    def _derive(self, llm: Any, **kw: Any) -> LoggingChatModel:
        return LoggingChatModel(llm, invoke_timeout=self.invoke_timeout, factory=self.factory, **kw)

    def bind_tools(self, tools: list, **kwargs: Any) -> LoggingChatModel:
        return self._derive(self.llm.bind_tools(tools, **kwargs), tools=tools)

    def with_structured_output(self, schema: Any, **kwargs: Any) -> LoggingChatModel:
        return self._derive(self.llm.bind_tools([schema]), structured_output=schema, tools=[schema])

    def with_retry(self, **kwargs: Any) -> LoggingChatModel:
        """Retries are the rollout's business (a retried call would record
        a second sample); the model is returned unchanged."""
        return self

    def with_config(self, config: Any = None, **kwargs: Any) -> LoggingChatModel:
        """Re-point at the current rollout's inference endpoint (the policy
        server moves to a new step between rollouts)."""
        rec = _CURRENT.get()
        if self.factory is not None and rec is not None:
            fresh = self.factory(rec.endpoint)
            if hasattr(self.llm, "bound"):  # a RunnableBinding around the client (bound tools)
                self.llm.bound = fresh
            else:
                self.llm = fresh
        elif hasattr(self.llm, "with_config"):
            self.llm = self.llm.with_config(config=config, **kwargs)
        return self


def wrap_rollout(model: Any, fn: Callable[..., Awaitable[Trajectory]],
                 log_dir: str | None = ".art/langgraph") -> Callable[..., Awaitable[Trajectory]]:
    """``fn`` run as a rollout against ``model``'s inference endpoint; the
    trajectory it returns is filled from the chat-model calls it made."""

    async def wrapper(*args: Any, **kwargs: Any) -> Trajectory:
        async def run() -> Trajectory:
            rec = start_rollout(model.inference_base_url, model.inference_api_key, model.inference_model_name,
                                log_dir)
            return fold_calls(rec, await fn(*args, **kwargs))

        # a copied context: this rollout's recorder is not seen by concurrent ones
        return await asyncio.get_running_loop().create_task(run(), context=contextvars.copy_context())

    return wrapper


def init_chat_model(model: Any = None, *, model_provider: str | None = None, configurable_fields: None = None,
                    config_prefix: str | None = None, invoke_timeout: float | None = DEFAULT_INVOKE_TIMEOUT,
                    **kwargs: Any) -> LoggingChatModel:
    """A logged chat model for the current rollout.  ``model`` may be an
    already built chat model (any provider) or a model name (default: the
    rollout's own model) for an OpenAI-compatible client pointed at the
    rollout's inference server; ``kwargs`` go to that client, and
    ``invoke_timeout`` bounds each asynchronous call."""
    if configurable_fields is not None:
        raise ValueError("configurable_fields is not supported")
    if config_prefix is not None:
        raise ValueError("config_prefix is not supported")
    if model is not None and not isinstance(model, str):
        return LoggingChatModel(model, invoke_timeout=invoke_timeout)
    if model_provider not in OPENAI_COMPATIBLE_PROVIDERS:
        raise ValueError(f"only OpenAI-compatible chat models are built here; pass a chat model instance to use "
                         f"provider {model_provider!r}")
    name = model

    def factory(endpoint: dict[str, Any]) -> Any:
        try:
            from langchain_openai import ChatOpenAI
        except ImportError as e:
            raise ImportError("init_chat_model() with a model name needs langchain_openai; pass a chat model "
                              "instance instead") from e
        kw = {"base_url": endpoint["base_url"], "api_key": endpoint["api_key"],
              "model": name or endpoint["model"], "temperature": 1.0}
        kw.update(kwargs)
        return ChatOpenAI(**kw)

    return LoggingChatModel(factory(current_recorder().endpoint), invoke_timeout=invoke_timeout, factory=factory)


__all__ = ["wrap_rollout", "init_chat_model", "LoggingChatModel", "RolloutRecorder", "convert_messages",
           "fold_calls", "to_openai_tool", "message_to_openai"]

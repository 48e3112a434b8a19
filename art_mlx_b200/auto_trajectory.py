"""Record the chat completions an agent makes into a Trajectory, without
changes to the agent's code.

Behaviour of the reference ``src/art/auto_trajectory.py:55-172``: inside
``capture_auto_trajectory(coro)`` (or ``with AutoTrajectoryContext()``),
every OpenAI-compatible chat-completion request sent through ``httpx`` (the
OpenAI SDK's transport) is recorded: the request's messages extend the
history they continue (the main one, or an additional history when the
conversation diverges, e.g. a sub-agent), followed by the returned choice
with its token ids.  Streamed responses are folded into one completion when
the stream ends.  ``auto_trajectory()`` returns the trajectory being
recorded, so a reward can be attached from inside the agent.

Mechanism here: ``httpx.Client.send`` / ``httpx.AsyncClient.send`` are
wrapped once; outside a capture context they are pass-through.  A streamed
body is wrapped in a recording byte stream that reports when it is closed.
"""

from __future__ import annotations

import contextvars
import json
from typing import Any, Coroutine

import httpx

from .trajectories import History, Trajectory

_ctx: contextvars.ContextVar["AutoTrajectoryContext"] = contextvars.ContextVar("art_auto_trajectory")


def auto_trajectory(*, required: bool = False) -> Trajectory | None:
    c = _ctx.get(None)
    if c is None:
        if required:
            raise RuntimeError("auto_trajectory(required=True) must run inside capture_auto_trajectory(...)")
        return None
    return c.trajectory


async def capture_auto_trajectory(coroutine: Coroutine[Any, Any, Any]) -> Trajectory:
    with AutoTrajectoryContext() as t:
        await coroutine
        return t


def _choice_from_payload(payload: dict[str, Any]):
    from openai.types.chat.chat_completion import Choice

    from .preprocessing.tokenize import attach_token_ids_to_choice

    choice = Choice.model_validate(payload["choices"][0])
    attach_token_ids_to_choice(choice, payload, 0)
    return choice


def _completion_from_sse(body: bytes):
    from openai.types.chat.chat_completion_chunk import ChatCompletionChunk

    from .openai import init_chat_completion, update_chat_completion

    completion = None
    for line in body.decode("utf-8", "replace").splitlines():
        line = line.strip()
        if not line.startswith("data:"):
            continue
        data = line[5:].strip()
        if not data or data == "[DONE]":
            continue
        chunk = ChatCompletionChunk.model_validate(json.loads(data))
        if completion is None:
            completion = init_chat_completion(chunk)
        update_chat_completion(completion, chunk)
    if completion is None:
        raise ValueError("no chunks in the streamed response")
    return completion


class AutoTrajectoryContext:
    def __init__(self) -> None:
        self.trajectory = Trajectory(messages_and_choices=[])

    def __enter__(self) -> Trajectory:
        _install()
        self._token = _ctx.set(self)
        return self.trajectory

    def __exit__(self, *exc: Any) -> None:
        _ctx.reset(self._token)
        self.trajectory.finish()

    # -------------------------------------------------------------- recording
    def record(self, request_body: bytes, response_body: bytes, streamed: bool) -> None:
        try:
            req = json.loads(request_body or b"{}")
        except (json.JSONDecodeError, UnicodeDecodeError):
            return
        messages = req.get("messages")
        if messages is None:
            return  # not a chat completion
        tools = req.get("tools")
        try:
            if streamed:
                completion = _completion_from_sse(response_body)
                payload = completion.model_dump(mode="python")
                choice = _choice_from_payload(payload)
            else:
                choice = _choice_from_payload(json.loads(response_body))
        except (ValueError, KeyError, json.JSONDecodeError):
            return
        hist = self._history_for(messages, tools)
        hist.messages_and_choices.extend(messages[len(hist.messages_and_choices):])
        hist.messages_and_choices.append(choice)
        hist.tools = tools

    def _history_for(self, messages: list, tools: Any) -> Trajectory | History:
        candidates: list[Trajectory | History] = [self.trajectory, *self.trajectory.additional_histories]
        for h in candidates:
            prior = h.messages()
            fresh = not prior and h.tools is None
            if prior == messages[: len(prior)] and (h.tools == tools or fresh):
                return h
        h = History(messages_and_choices=[])
        self.trajectory.additional_histories.append(h)
        return h


class _RecordingStream(httpx.AsyncByteStream, httpx.SyncByteStream):
    def __init__(self, inner: Any, on_done) -> None:
        self._inner, self._on_done, self._buf, self._done = inner, on_done, bytearray(), False

    def _finish(self) -> None:
        if not self._done:
            self._done = True
            self._on_done(bytes(self._buf))

    async def __aiter__(self):
        async for chunk in self._inner:
            self._buf += chunk
            yield chunk
        self._finish()

    def __iter__(self):
        for chunk in self._inner:
            self._buf += chunk
            yield chunk
        self._finish()

    async def aclose(self) -> None:
        await self._inner.aclose()
        self._finish()

    def close(self) -> None:
        self._inner.close()
        self._finish()


_installed = False


def _install() -> None:
    global _installed
    if _installed:
        return
    _installed = True
    orig_async, orig_sync = httpx.AsyncClient.send, httpx.Client.send

    def hook(request: httpx.Request, response: httpx.Response, ctx: AutoTrajectoryContext) -> None:
        body = request.content
        streamed = b'"stream": true' in body or b'"stream":true' in body
        if response.is_stream_consumed or hasattr(response, "_content"):
            ctx.record(body, response.content, streamed)
        else:
            response.stream = _RecordingStream(response.stream, lambda data: ctx.record(body, data, streamed))

    async def send_async(self, request, *args, **kwargs):
        response = await orig_async(self, request, *args, **kwargs)
        ctx = _ctx.get(None)
        if ctx is not None and request.url.path.endswith("/chat/completions"):
            hook(request, response, ctx)
        return response

    def send_sync(self, request, *args, **kwargs):
        response = orig_sync(self, request, *args, **kwargs)
        ctx = _ctx.get(None)
        if ctx is not None and request.url.path.endswith("/chat/completions"):
            hook(request, response, ctx)
        return response

    httpx.AsyncClient.send = send_async  # type: ignore[method-assign]
    httpx.Client.send = send_sync  # type: ignore[method-assign]

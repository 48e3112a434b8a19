"""Streaming helpers for OpenAI-compatible chat completions.

Same contract as the reference ``src/art/openai.py:16-167``:
``consume_chat_completion_stream`` (async) and
``consume_sync_chat_completion_stream`` fold a stream of
``ChatCompletionChunk`` objects into the ``ChatCompletion`` a non-streaming
call would have returned (content, tool calls assembled from their argument
fragments, per-token logprobs, finish reasons), so a streamed rollout can be
recorded in a ``Trajectory``.  ``on_chunk(chunk, completion_so_far)`` may
raise ``StopIteration`` to close the stream early.
"""

from __future__ import annotations

from typing import Any, Callable

from openai.types.chat.chat_completion import ChatCompletion, Choice, ChoiceLogprobs
from openai.types.chat.chat_completion_chunk import ChatCompletionChunk
from openai.types.chat.chat_completion_message import ChatCompletionMessage


def init_chat_completion(chunk: ChatCompletionChunk) -> ChatCompletion:
    return ChatCompletion(
        id=chunk.id, created=chunk.created, model=chunk.model, object="chat.completion",
        choices=[
            Choice(finish_reason="stop", index=c.index, logprobs=ChoiceLogprobs() if c.logprobs else None,
                   message=ChatCompletionMessage(role="assistant"))
            for c in chunk.choices
        ],
    )


def _choice(completion: ChatCompletion, index: int) -> Choice:
    for c in completion.choices:
        if c.index == index:
            return c
    c = Choice(finish_reason="stop", index=index, logprobs=None, message=ChatCompletionMessage(role="assistant"))
    completion.choices.append(c)
    return c


def update_chat_completion(completion: ChatCompletion, chunk: ChatCompletionChunk) -> None:
    """Fold one chunk into ``completion`` in place."""
    from openai.types.chat.chat_completion_message_function_tool_call import (
        ChatCompletionMessageFunctionToolCall,
        Function,
    )

    if chunk.usage is not None:
        completion.usage = chunk.usage
    chunk_extra = getattr(chunk, "model_extra", None) or {}
    if chunk_extra.get("prompt_token_ids") is not None:  # rollout servers report the prompt ids
        ext = completion.__pydantic_extra__ if completion.__pydantic_extra__ is not None else {}
        ext["prompt_token_ids"] = list(chunk_extra["prompt_token_ids"])
        object.__setattr__(completion, "__pydantic_extra__", ext)
    for delta_choice in chunk.choices:
        c = _choice(completion, delta_choice.index)
        d = delta_choice.delta
        msg = c.message
        if d.content:
            msg.content = (msg.content or "") + d.content
        if getattr(d, "refusal", None):
            msg.refusal = (msg.refusal or "") + d.refusal
        if d.role:
            msg.role = d.role
        for tc in d.tool_calls or []:
            calls = list(msg.tool_calls or [])
            while len(calls) <= tc.index:
                calls.append(ChatCompletionMessageFunctionToolCall(
                    id="", type="function", function=Function(name="", arguments="")))
            call = calls[tc.index]
            if tc.id:
                call.id = tc.id
            if tc.function is not None:
                if tc.function.name:
                    call.function.name += tc.function.name
                if tc.function.arguments:
                    call.function.arguments += tc.function.arguments
            msg.tool_calls = calls
        if delta_choice.logprobs is not None:
            if c.logprobs is None:
                c.logprobs = ChoiceLogprobs()
            if delta_choice.logprobs.content:
                c.logprobs.content = list(c.logprobs.content or []) + list(delta_choice.logprobs.content)
            if delta_choice.logprobs.refusal:
                c.logprobs.refusal = list(c.logprobs.refusal or []) + list(delta_choice.logprobs.refusal)
        if delta_choice.finish_reason:
            c.finish_reason = delta_choice.finish_reason
        extra = getattr(delta_choice, "model_extra", None) or {}
        if extra.get("token_ids"):  # servers that stream token ids (rollout servers)
            ce = c.__pydantic_extra__ if c.__pydantic_extra__ is not None else {}
            ce["token_ids"] = list(ce.get("token_ids") or []) + list(extra["token_ids"])
            object.__setattr__(c, "__pydantic_extra__", ce)


async def consume_chat_completion_stream(
    stream: Any, on_chunk: Callable[[ChatCompletionChunk, ChatCompletion], Any] | None = None
) -> ChatCompletion:
    completion: ChatCompletion | None = None
    async for chunk in stream:
        if completion is None:
            completion = init_chat_completion(chunk)
        update_chat_completion(completion, chunk)
        if on_chunk is not None:
            try:
                on_chunk(chunk, completion)
            except StopIteration:
                await stream.close()
                break
    if completion is None:
        raise ValueError("the stream produced no chunks")
    return completion


def consume_sync_chat_completion_stream(stream: Any) -> ChatCompletion:
    completion: ChatCompletion | None = None
    for chunk in stream:
        if completion is None:
            completion = init_chat_completion(chunk)
        update_chat_completion(completion, chunk)
    if completion is None:
        raise ValueError("the stream produced no chunks")
    return completion

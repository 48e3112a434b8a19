"""Agent rollout in a tau-bench environment.

The policy (an OpenAI-compatible endpoint, usually ``model.openai_client()``
of a registered :class:`TrainableModel`) talks to the environment: the
system message is the domain policy, the first user turn the environment's
observation; a tool call becomes the action ``name(k=v, ...)`` (arguments
in Python ``repr``, the environment's action syntax), plain text is a reply
to the simulated user.  Step rewards add up into the trajectory's reward;
the episode ends when the environment terminates, after ``max_turns`` or
when the next completion would overflow ``context_limit`` tokens.
"""

from __future__ import annotations

import json
import os
from typing import Any

from ..trajectories import Trajectory
from .client import Scenario, TauBenchClient, default_client

DEFAULT_MAX_COMPLETION_TOKENS = 4096


def tool_call_action(tool_call: Any) -> str:
    fn = tool_call.function if hasattr(tool_call, "function") else tool_call["function"]
    name = fn.name if hasattr(fn, "name") else fn["name"]
    raw = fn.arguments if hasattr(fn, "arguments") else fn["arguments"]
    args = json.loads(raw or "{}")
    return f"{name}({', '.join(f'{k}={v!r}' for k, v in args.items())})"


def default_user_llm_args(user_model_name: str) -> dict[str, Any]:
    """Greedy user simulator; the API key of the user model's provider is
    forwarded when set in the environment."""
    args: dict[str, Any] = {"temperature": 0.0}
    m = user_model_name.lower()
    env = None
    if m.startswith("openrouter/"):
        env = "OPENROUTER_API_KEY"
    elif m.startswith(("openai/", "gpt-", "o1", "o3", "o4")):
        env = "OPENAI_API_KEY"
    elif m.startswith(("anthropic/", "claude")):
        env = "ANTHROPIC_API_KEY"
    elif m.startswith(("gemini/", "google/")):
        env = "GEMINI_API_KEY" if os.getenv("GEMINI_API_KEY") else "GOOGLE_API_KEY"
    if env and os.getenv(env):
        args["api_key"] = os.environ[env]
    return args


async def rollout(scenario: Scenario, policy: Any, *, model_name: str | None = None, client: TauBenchClient | None = None,
                  max_turns: int | None = None, chat_completion_kwargs: dict[str, Any] | None = None,
                  user_model_name: str = "gpt-4.1-2025-04-14", user_chat_completion_kwargs: dict[str, Any] | None = None,
                  context_limit: int = 32768, retrieval_config: str | None = None,
                  retrieval_config_kwargs: dict[str, Any] | None = None) -> Trajectory:
    """``policy`` is a :class:`~art_mlx_b200.model.Model` (its OpenAI client
    and inference name are used) or an ``AsyncOpenAI``-like client together
    with ``model_name``."""
    client = client or default_client()
    if hasattr(policy, "openai_client") and hasattr(policy, "get_inference_name"):
        oa, name = policy.openai_client(), policy.get_inference_name()
    else:
        if model_name is None:
            raise TypeError("model_name is required with a plain OpenAI client")
        oa, name = policy, model_name
    kw = dict(chat_completion_kwargs or {})
    want = int(kw.get("max_tokens") or kw.get("max_completion_tokens") or DEFAULT_MAX_COMPLETION_TOKENS)
    async with client.environment(domain=scenario.domain, task_id=scenario.task.id, user_llm=user_model_name,
                                  user_llm_args=user_chat_completion_kwargs or default_user_llm_args(user_model_name),
                                  retrieval_config=retrieval_config,
                                  retrieval_config_kwargs=retrieval_config_kwargs) as env:
        traj = Trajectory(
            messages_and_choices=[{"role": "system", "content": env.info.get("policy", "")},
                                  {"role": "user", "content": env.observation.removeprefix("user: ")}],
            tools=env.info.get("tools"), reward=0.0, metrics={"cost/user": 0.0},
            metadata={"scenario_id": scenario.task.id},
        )
        turns, done = 0, False
        while not done and (max_turns is None or turns < max_turns):
            comp = await oa.chat.completions.create(messages=traj.messages(), model=name, stream=False,
                                                    tool_choice="auto", tools=traj.tools or [], **kw)
            choice = comp.choices[0]
            traj.messages_and_choices.append(choice)
            calls = getattr(choice.message, "tool_calls", None)
            if calls:
                for call in calls:
                    step = await client.step_environment(env.id, tool_call_action(call))
                    traj.messages_and_choices.append({"role": "tool", "tool_call_id": call.id,
                                                      "content": step.observation.removeprefix("tool: ")})
                    traj.reward += step.reward
                    done = step.terminated
            else:
                step = await client.step_environment(env.id, choice.message.content or "")
                traj.metrics["cost/user"] += float(step.info.get("user_message_cost", 0.0))
                traj.messages_and_choices.append({"role": "user",
                                                  "content": step.observation.removeprefix("user: ")})
                traj.reward += step.reward
                done = step.terminated
            turns += 1
            usage = getattr(comp, "usage", None)
            if usage is not None and getattr(usage, "total_tokens", 0) + want > context_limit:
                break
        traj.metrics["num_turns"] = turns
        return traj

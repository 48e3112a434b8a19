"""Synthetic rollouts in the rollout server's wire format.

Builds ``TrajectoryGroup`` objects whose trainable ``Choice`` objects carry
``prompt_token_ids`` / ``token_ids`` and per-token sampled logprobs exactly
as the OpenAI-compatible server returns them, so the whole public training
path (tokenize → advantages → prefix-tree pack → train) runs without a
server.  Used by the benchmark and the tests (there is no network for
datasets here).
"""

from __future__ import annotations

import random
from typing import Literal

from ..trajectories import Trajectory, TrajectoryGroup


def make_choice(prompt_ids: list[int], completion_ids: list[int], logprobs: list[float]):
    """A ``Choice`` carrying rollout token ids and logprobs (validation-free
    construction: these objects are produced in bulk)."""
    from openai.types.chat.chat_completion import Choice, ChoiceLogprobs
    from openai.types.chat.chat_completion_message import ChatCompletionMessage
    from openai.types.chat.chat_completion_token_logprob import ChatCompletionTokenLogprob

    content = [
        ChatCompletionTokenLogprob.model_construct(token=f"t{t}", logprob=lp, bytes=None, top_logprobs=[])
        for t, lp in zip(completion_ids, logprobs)
    ]
    choice = Choice.model_construct(
        finish_reason="stop",
        index=0,
        logprobs=ChoiceLogprobs.model_construct(content=content, refusal=None),
        message=ChatCompletionMessage.model_construct(role="assistant", content="", tool_calls=None),
    )
    object.__setattr__(
        choice,
        "__pydantic_extra__",
        {"prompt_token_ids": list(prompt_ids), "token_ids": list(completion_ids)},
    )
    return choice


def synthetic_groups(
    *,
    num_groups: int,
    rollouts_per_group: int,
    prompt_len: int,
    completion_len: int,
    vocab_size: int,
    seed: int = 0,
    reward: Literal["normal", "bernoulli"] = "normal",
) -> list[TrajectoryGroup]:
    """``num_groups`` groups; each group shares one uniform-random prompt of
    ``prompt_len`` tokens and has ``rollouts_per_group`` completions of
    ``completion_len`` uniform-random tokens with rewards N(0,1) or
    Bernoulli(0.5).  Sampled logprobs are drawn in [-4, -0.01]."""
    rng = random.Random(seed)
    groups = []
    for _ in range(num_groups):
        prompt = [rng.randrange(vocab_size) for _ in range(prompt_len)]
        trajs = []
        rewards = []
        for k in range(rollouts_per_group):
            comp = [rng.randrange(vocab_size) for _ in range(completion_len)]
            lps = [-rng.uniform(0.01, 4.0) for _ in range(completion_len)]
            if reward == "normal":
                r = rng.gauss(0.0, 1.0)
            else:
                r = float(rng.random() < 0.5)
            rewards.append(r)
            trajs.append(
                Trajectory(
                    messages_and_choices=[
                        {"role": "user", "content": "synthetic"},
                        make_choice(prompt, comp, lps),
                    ],
                    reward=r,
                )
            )
        if reward == "bernoulli" and len(set(rewards)) == 1:
            # keep every group trainable: flip one reward of a degenerate group
            trajs[0].reward = 1.0 - trajs[0].reward
        groups.append(TrajectoryGroup(trajs))
    return groups

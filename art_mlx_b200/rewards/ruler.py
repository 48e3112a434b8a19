"""RULER: relative rewards from an LLM judge.

Behaviour of the reference ``src/art/rewards/ruler.py:86`` (``ruler``) and
``:266`` (``ruler_score_group``): all trajectories of one group are shown to
a judge model together (a message prefix shared by all of them is sent once
as context; a group of identical trajectories is sent as one), the judge
returns one score in [0, 1] per trajectory, and ``ruler_score_group`` puts
those scores in as rewards, keeping the original reward in
``metrics["independent_reward"]`` and the score in ``metrics["ruler_score"]``.
GRPO normalises rewards inside a group, so relative judgements are all it
needs.

The judge is any OpenAI-compatible chat endpoint: ``client`` (an
``openai.AsyncOpenAI``-like object, e.g. ``model.openai_client()`` of a
model served by this framework's rollout server) or, by default, an
``AsyncOpenAI`` client configured from the environment.  ``judge_model``
may carry a ``provider/`` prefix, which is dropped for the request.
"""

from __future__ import annotations

import json
from typing import Any

from pydantic import BaseModel, Field

from ..trajectories import Trajectory, TrajectoryGroup


class TrajectoryScore(BaseModel):
    trajectory_id: str = Field(description="id of the scored trajectory")
    explanation: str = Field(description="one or two sentences on how the trajectory did")
    score: float = Field(description="score in [0, 1]")


class JudgeResponse(BaseModel):
    scores: list[TrajectoryScore]


DEFAULT_RUBRIC = """\
- Reaching the goal always scores clearly above not reaching it.
- Among trajectories that reach the goal, the more direct one (fewer wasted steps) scores higher.
- Score gaps should track quality gaps: small for near-equal trajectories, large for clear differences.
- Partial progress toward the goal earns partial credit."""


def _shared_prefix_len(message_lists: list[list[Any]]) -> int:
    n = 0
    for i, m in enumerate(message_lists[0]):
        if all(len(ml) > i and ml[i] == m for ml in message_lists):
            n += 1
        else:
            break
    return n


def build_judge_messages(message_lists: list[list[Any]], rubric: str = DEFAULT_RUBRIC,
                         tools: list[dict] | None = None) -> tuple[list[dict[str, str]], bool]:
    """The judge conversation, and whether the trajectories were identical
    (then only one is shown and its score is reused for all)."""
    shared = _shared_prefix_len(message_lists)
    identical = len(message_lists) > 1 and all(len(ml) == shared for ml in message_lists)
    parts: list[str] = []
    if shared and not identical:
        parts.append("<context>\n" + json.dumps(message_lists[0][:shared], default=str) + "\n</context>")
    if tools:
        parts.append("<available_tools>\n" + json.dumps(tools, default=str) + "\n</available_tools>")
    shown = [message_lists[0]] if identical else [ml[shared:] for ml in message_lists]
    body = "\n\n".join(
        f'<trajectory id="{i}">\n{json.dumps(ml, default=str)}\n</trajectory>' for i, ml in enumerate(shown, 1)
    )
    parts.append("Trajectories:\n\n" + body)
    system = (
        "Each trajectory below was produced by an agent pursuing the same goal. Infer that goal, judge "
        "every trajectory against it and give each a score between 0 and 1.\n\nRubric:\n" + rubric +
        '\n\nAnswer with JSON only: {"scores": [{"trajectory_id": "<id>", "explanation": "...", "score": <0..1>}, ...]}'
    )
    return [{"role": "system", "content": system}, {"role": "user", "content": "\n\n".join(parts)}], identical


def _default_client() -> Any:
    from openai import AsyncOpenAI

    return AsyncOpenAI()


async def ruler(
    message_lists: list[list[Any]],
    judge_model: str = "openai/o3",
    extra_params: dict[str, Any] | None = None,
    rubric: str = DEFAULT_RUBRIC,
    tools: list[dict] | None = None,
    *,
    client: Any | None = None,
    debug: bool = False,
) -> list[TrajectoryScore]:
    """Scores for each message list (same order)."""
    if not message_lists:
        return []
    messages, identical = build_judge_messages(message_lists, rubric, tools)
    client = client or _default_client()
    model = judge_model.split("/", 1)[1] if "/" in judge_model else judge_model
    resp = await client.chat.completions.create(
        model=model, messages=messages, response_format={"type": "json_object"}, **(extra_params or {})
    )
    if not resp.choices:
        raise ValueError("judge returned no choices")
    content = resp.choices[0].message.content or "{}"
    if debug:
        print("[RULER] judge answer:", content)
    parsed = JudgeResponse.model_validate_json(content)
    if identical:
        if len(parsed.scores) != 1:
            raise ValueError(f"expected 1 score for identical trajectories, got {len(parsed.scores)}")
        return [parsed.scores[0].model_copy(update={"trajectory_id": str(i)})
                for i in range(1, len(message_lists) + 1)]
    if len(parsed.scores) != len(message_lists):
        raise ValueError(f"expected {len(message_lists)} scores, got {len(parsed.scores)}")
    return parsed.scores


async def ruler_score_group(
    group: TrajectoryGroup,
    judge_model: str = "openai/o3",
    extra_params: dict[str, Any] | None = None,
    rubric: str = DEFAULT_RUBRIC,
    *,
    client: Any | None = None,
    swallow_exceptions: bool = False,
    debug: bool = False,
) -> TrajectoryGroup | None:
    """A copy of ``group`` with the judge's scores as rewards (``None`` on a
    judge error when ``swallow_exceptions``)."""
    for t in group.trajectories:
        if t.additional_histories:
            raise ValueError("trajectories with additional histories cannot be judged yet")
    trajs: list[Trajectory] = [t.model_copy(deep=True) for t in group.trajectories]
    message_lists = [t.messages() for t in trajs]
    try:
        scores = await ruler(message_lists, judge_model, extra_params, rubric,
                             tools=trajs[0].tools if trajs else None, client=client, debug=debug)
    except Exception:
        if swallow_exceptions:
            return None
        raise
    for t, s in zip(trajs, scores):
        t.metrics["independent_reward"] = t.reward
        t.metrics["ruler_score"] = s.score
        t.reward = s.score
        t.log(f"RULER explanation: {s.explanation}")
    return TrajectoryGroup(trajs, exceptions=list(group.exceptions), metadata=dict(group.metadata),
                           metrics=dict(group.metrics), logs=list(group.logs))

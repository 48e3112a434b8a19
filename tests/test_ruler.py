"""RULER with a fake OpenAI-compatible judge."""

import asyncio
import json
from types import SimpleNamespace

import pytest

from art_mlx_b200.rewards import ruler, ruler_score_group
from art_mlx_b200.rewards.ruler import build_judge_messages
from art_mlx_b200.trajectories import Trajectory, TrajectoryGroup


class FakeJudge:
    def __init__(self, scores):
        self.scores = scores
        self.seen = []
        self.chat = SimpleNamespace(completions=SimpleNamespace(create=self.create))

    async def create(self, model, messages, **kw):
        self.seen.append((model, messages, kw))
        body = {"scores": [{"trajectory_id": str(i + 1), "explanation": "ok", "score": s}
                           for i, s in enumerate(self.scores)]}
        msg = SimpleNamespace(content=json.dumps(body))
        return SimpleNamespace(choices=[SimpleNamespace(message=msg)])


def _traj(answer, reward=0.0):
    return Trajectory(messages_and_choices=[{"role": "system", "content": "be right"},
                                            {"role": "user", "content": "2+2?"},
                                            {"role": "assistant", "content": answer}], reward=reward)


def test_shared_prefix_sent_once_and_identical_groups_collapse():
    msgs, identical = build_judge_messages([_traj("4").messages(), _traj("5").messages()])
    assert not identical
    user = msgs[1]["content"]
    assert user.count("be right") == 1 and "<context>" in user and 'id="2"' in user
    msgs, identical = build_judge_messages([_traj("4").messages(), _traj("4").messages()])
    assert identical and 'id="2"' not in msgs[1]["content"]


def test_ruler_score_group_sets_rewards():
    judge = FakeJudge([0.9, 0.1])
    g = TrajectoryGroup([_traj("4", 1.0), _traj("5", 0.0)])
    out = asyncio.run(ruler_score_group(g, "openai/some-judge", client=judge))
    assert [t.reward for t in out] == [0.9, 0.1]
    assert out.trajectories[0].metrics["independent_reward"] == 1.0
    assert out.trajectories[1].metrics["ruler_score"] == 0.1
    assert g.trajectories[0].reward == 1.0  # the input group is untouched
    assert judge.seen[0][0] == "some-judge"


def test_ruler_errors():
    judge = FakeJudge([0.5])  # wrong number of scores
    g = TrajectoryGroup([_traj("4"), _traj("5")])
    with pytest.raises(ValueError, match="expected 2 scores"):
        asyncio.run(ruler([t.messages() for t in g], client=judge))
    assert asyncio.run(ruler_score_group(g, client=judge, swallow_exceptions=True)) is None

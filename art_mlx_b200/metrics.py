"""Metric summaries and the cumulative metrics builder.

Mirrors the reference's taxonomy (``src/art/metrics.py:77-409``,
``metrics_taxonomy.py``): per-step group summaries (reward mean/std,
exceptions, trainable groups), ``data/step_trainer_tokens``, cumulative
``data/cum/trainer_tokens`` and ``throughput/avg_trainer_tok_per_s``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Iterable

from .trajectories import TrajectoryGroup

TRAIN_GRADIENT_STEPS_KEY = "data/step_num_gradient_steps"


def summarize_groups(groups: Iterable[TrajectoryGroup]) -> dict[str, float]:
    groups = list(groups)
    rewards = [t.reward for g in groups for t in g]
    out: dict[str, float] = {
        "num_groups": float(len(groups)),
        "num_trajectories": float(len(rewards)),
        "exceptions": float(sum(len(g.exceptions) for g in groups)),
    }
    if rewards:
        mean = sum(rewards) / len(rewards)
        out["reward"] = mean
        out["reward_std_dev"] = math.sqrt(sum((r - mean) ** 2 for r in rewards) / len(rewards))
    trainable = 0
    for g in groups:
        rs = [t.reward for t in g]
        if len(rs) > 1 and max(rs) != min(rs):
            trainable += 1
    out["num_groups_trainable"] = float(trainable)
    metric_sums: dict[str, list[float]] = {}
    for g in groups:
        for t in g:
            for k, v in t.metrics.items():
                metric_sums.setdefault(k, []).append(float(v))
    for k, vals in metric_sums.items():
        out[k] = sum(vals) / len(vals)
    return out


@dataclass
class MetricsBuilder:
    """Accumulates cumulative counters across steps (tokens, seconds)."""

    cum: dict[str, float] = field(default_factory=dict)

    def update(self, step_metrics: dict[str, float]) -> dict[str, float]:
        out = dict(step_metrics)
        tok = step_metrics.get("data/step_trainer_tokens")
        sec = step_metrics.get("time/step_trainer_s")
        if tok is not None:
            self.cum["data/cum/trainer_tokens"] = self.cum.get("data/cum/trainer_tokens", 0.0) + tok
        if sec is not None:
            self.cum["time/cum/trainer_s"] = self.cum.get("time/cum/trainer_s", 0.0) + sec
        out.update(self.cum)
        tt, ts = self.cum.get("data/cum/trainer_tokens"), self.cum.get("time/cum/trainer_s")
        if tt is not None and ts:
            out["throughput/avg_trainer_tok_per_s"] = tt / ts
        if tok is not None and sec:
            out["throughput/step_trainer_tok_per_s"] = tok / sec
        return out

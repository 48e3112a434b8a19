"""Checkpoint retention for the pipeline trainer (same contract as the
reference ``src/art/pipeline_trainer/checkpoint_retention.py``): a strategy
receives the checkpoints that are eligible for deletion and returns the
steps to keep."""

from __future__ import annotations

from collections.abc import Callable, Iterable
from datetime import datetime

from pydantic import BaseModel, Field

CHECKPOINT_CREATED_AT_METRIC = "checkpoint/created_at_unix"
CHECKPOINT_EVAL_COMPLETED_METRIC = "checkpoint/eval_completed"
CHECKPOINT_SAVED_METRIC = "checkpoint/saved"


class CheckpointInfo(BaseModel):
    step: int
    path: str
    created_at: datetime
    is_eval_step: bool = False
    metrics: dict[str, float] = Field(default_factory=dict)


class CheckpointRetentionContext(BaseModel):
    current_step: int
    checkpoints: list[CheckpointInfo] = Field(default_factory=list)


CheckpointRetentionStrategy = Callable[[CheckpointRetentionContext], Iterable[int]]


def keep_recent_and_top(*, recent: int = 5, top: int = 2, metric: str = "val/reward") -> CheckpointRetentionStrategy:
    """Keep the ``recent`` newest eligible checkpoints plus the ``top`` best
    by ``metric`` (ties broken by the later step)."""
    if recent < 0 or top < 0:
        raise ValueError("recent and top must be >= 0")

    def strategy(ctx: CheckpointRetentionContext) -> set[int]:
        steps = sorted(c.step for c in ctx.checkpoints)
        keep = set(steps[-recent:]) if recent else set()
        scored = sorted((c for c in ctx.checkpoints if metric in c.metrics),
                        key=lambda c: (c.metrics[metric], c.step), reverse=True)
        keep.update(c.step for c in scored[:top])
        return keep & set(steps)

    return strategy

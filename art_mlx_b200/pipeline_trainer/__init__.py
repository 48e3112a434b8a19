"""Asynchronous rollout / training / evaluation pipeline."""

from .checkpoint_retention import (
    CheckpointInfo,
    CheckpointRetentionContext,
    CheckpointRetentionStrategy,
    keep_recent_and_top,
)
from .trainer import PipelineState, PipelineTrainer, make_group_rollout_fn

__all__ = [
    "CheckpointInfo",
    "CheckpointRetentionContext",
    "CheckpointRetentionStrategy",
    "PipelineState",
    "PipelineTrainer",
    "keep_recent_and_top",
    "make_group_rollout_fn",
]

"""Reward helpers."""

from .ruler import DEFAULT_RUBRIC, TrajectoryScore, ruler, ruler_score_group

__all__ = ["DEFAULT_RUBRIC", "TrajectoryScore", "ruler", "ruler_score_group"]

"""Slicing packed tensors into per-micro-step train inputs.

Reference ``src/art/preprocessing/inputs.py:19-50``: one packed row per
micro step; the warm-up micro keeps only the first 1024 tokens and runs at a
negligible learning rate with no KL.
"""

from __future__ import annotations

from typing import Any

import torch

from ..types import TrainConfig
from .pack import PackedTensors


def create_train_inputs(
    packed_tensors: PackedTensors,
    offset: int,
    config: TrainConfig,
    _config: dict[str, Any],
    warmup: bool,
) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for key, value in packed_tensors.items():
        if isinstance(value, torch.Tensor):
            row = value[offset : offset + 1]
            out[key] = row[:, :1024] if warmup and value.dim() > 1 else row
    out["pixel_values"] = [None]
    out["image_grid_thw"] = [None]
    out["config"] = (
        config.model_copy(update={"learning_rate": 1e-9, "kl_penalty_coef": 0.0})
        if warmup
        else config
    )
    out["_config"] = _config
    out["return_new_logprobs"] = False
    return out

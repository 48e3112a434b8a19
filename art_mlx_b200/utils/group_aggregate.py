"""Group-wise reductions over the token axis of ``[B, S, *F]`` tensors.

Same contract as the reference ``src/art/utils/group_aggregate.py:8-146``:
``by`` labels each ``(b, s)`` token with a categorical group id (ids are
shared across the whole batch); the reduction is taken per ``(b, group)`` and
is either broadcast back to token shape or returned compactly as
``[B, num_groups, *F]``.  Implemented with ``index_add_`` over a flattened
``b * G + g`` index, which is differentiable w.r.t. ``values``.
"""

from __future__ import annotations

from typing import Literal

import torch

Reduction = Literal["sum", "mean", "var", "std", "count", "min", "max"]


def group_aggregate(
    values: torch.Tensor,
    *,
    by: torch.Tensor,
    reduce: Reduction = "mean",
    eps: float = 1e-8,
    broadcast: bool = True,
) -> torch.Tensor:
    if values.dim() < 2:
        raise ValueError("`values` must have at least 2 dimensions [B, S].")
    if tuple(by.shape[:2]) != tuple(values.shape[:2]):
        raise ValueError("`by` must match the first two dimensions of `values` (B, S).")
    B, S = values.shape[:2]
    feat = tuple(values.shape[2:])
    if values.numel() == 0:
        if broadcast:
            return values.clone()
        return values.new_empty((B, 0, *feat))
    if by.numel() == 0:
        raise ValueError("`by` cannot be empty when values is non-empty")

    _, inverse = torch.unique(by.reshape(B, S), return_inverse=True)
    G = int(inverse.max().item()) + 1
    flat_values = values.reshape(B * S, -1)
    P = flat_values.shape[1]
    slot = (
        torch.arange(B, device=values.device).unsqueeze(1) * G + inverse.reshape(B, S)
    ).reshape(-1)

    def scatter_sum(v: torch.Tensor) -> torch.Tensor:
        out = v.new_zeros(B * G, v.shape[1])
        return out.index_add(0, slot, v)

    if reduce in ("min", "max"):
        fill = float("inf") if reduce == "min" else float("-inf")
        agg = flat_values.new_full((B * G, P), fill)
        agg = agg.scatter_reduce(
            0, slot.unsqueeze(1).expand(-1, P), flat_values, reduce="amin" if reduce == "min" else "amax"
        )
    elif reduce == "sum":
        agg = scatter_sum(flat_values)
    else:
        counts = scatter_sum(torch.ones_like(flat_values[:, :1]))
        if reduce == "count":
            agg = counts.expand(-1, P)
        else:
            sums = scatter_sum(flat_values)
            mean = sums / (counts + eps)
            if reduce == "mean":
                agg = mean
            elif reduce in ("var", "std"):
                sq = scatter_sum(flat_values * flat_values) / (counts + eps)
                var = torch.clamp(sq - mean * mean, min=0.0)
                agg = var if reduce == "var" else torch.sqrt(var + eps)
            else:
                raise ValueError(f"Unsupported reduce type: {reduce}")

    if broadcast:
        return agg.index_select(0, slot).reshape(values.shape)
    return agg.reshape(B, G, *feat)

"""Hand a Trajectory out of a coroutine that returns something else
(reference ``src/art/yield_trajectory.py``): the agent calls
``yield_trajectory(t)``; ``capture_yielded_trajectory(coro)`` runs it and
returns the last trajectory yielded inside it."""

from __future__ import annotations

import contextvars
from typing import Any, Coroutine

from .trajectories import Trajectory


class _Slot:
    def __init__(self) -> None:
        self.trajectory: Trajectory | None = None


_slot: contextvars.ContextVar[_Slot | None] = contextvars.ContextVar("art_yield_trajectory", default=None)


def yield_trajectory(trajectory: Trajectory) -> None:
    s = _slot.get()
    if s is None:
        raise RuntimeError("yield_trajectory() must run inside capture_yielded_trajectory(...)")
    s.trajectory = trajectory


async def capture_yielded_trajectory(coroutine: Coroutine[Any, Any, Any]) -> Trajectory:
    slot = _Slot()
    token = _slot.set(slot)
    try:
        await coroutine
    finally:
        _slot.reset(token)
    if slot.trajectory is None:
        raise RuntimeError("no trajectory was yielded")
    return slot.trajectory

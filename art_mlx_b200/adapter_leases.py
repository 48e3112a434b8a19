"""Pinning the inference step and leasing adapters.

Reference ``src/art/adapter_leases.py:1-26`` and ``local/adapter_leases.py``:
``pin_inference_step(name, step)`` makes ``model.get_inference_name()``
resolve to ``{name}@{step}`` inside the context (a rollout keeps sampling
from one checkpoint while training moves on), and an
:class:`AdapterLeaseManager` counts users of each step so checkpoint
cleanup keeps every leased step.
"""

from __future__ import annotations

import asyncio
from collections import Counter
from contextlib import asynccontextmanager
from contextvars import ContextVar
from typing import AsyncIterator

_pinned: ContextVar[dict[str, int] | None] = ContextVar("art_pinned_inference_steps", default=None)


def pinned_inference_step(model_name: str) -> int | None:
    return (_pinned.get() or {}).get(model_name)


@asynccontextmanager
async def pin_inference_step(model_name: str, step: int) -> AsyncIterator[None]:
    steps = dict(_pinned.get() or {})
    steps[model_name] = step
    token = _pinned.set(steps)
    try:
        yield
    finally:
        _pinned.reset(token)


class AdapterLeaseManager:
    def __init__(self) -> None:
        self._counts: Counter[int] = Counter()
        self._cond = asyncio.Condition()

    @asynccontextmanager
    async def lease(self, step: int) -> AsyncIterator[None]:
        async with self._cond:
            self._counts[step] += 1
        try:
            yield
        finally:
            async with self._cond:
                self._counts[step] -= 1
                if self._counts[step] <= 0:
                    del self._counts[step]
                self._cond.notify_all()

    def active_steps(self) -> set[int]:
        return set(self._counts)

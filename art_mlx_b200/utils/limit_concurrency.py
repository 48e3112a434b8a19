"""Cap the number of concurrent calls of an async function.

Interface of the reference's ``src/art/utils/limit_concurrency.py``: at most
``n`` calls run at once, per key when ``derive_key(*args, **kwargs)`` is
given (e.g. one limit per judge model), else one shared limit.
"""

from __future__ import annotations

import asyncio
import functools
from typing import Any, Callable, Optional


def limit_concurrency(n: int, derive_key: Optional[Callable[..., str]] = None):
    if n < 1:
        raise ValueError("n must be >= 1")

    def decorator(func):
        sems: dict[tuple[int, str], asyncio.Semaphore] = {}

        @functools.wraps(func)
        async def wrapper(*args: Any, **kwargs: Any) -> Any:
            key = derive_key(*args, **kwargs) if derive_key is not None else "default"
            # one semaphore per (event loop, key): a semaphore is bound to its loop
            loop_key = (id(asyncio.get_running_loop()), key)
            sem = sems.get(loop_key)
            if sem is None:
                sem = sems[loop_key] = asyncio.Semaphore(n)
            async with sem:
                return await func(*args, **kwargs)

        return wrapper

    return decorator

"""Retry with exponential backoff for sync and async callables.

Same interface as the reference's ``src/art/utils/retry.py`` (``retry(max_attempts,
delay, backoff_factor, exceptions, on_retry)``): rollouts and judge calls
wrap flaky network requests with it.
"""

from __future__ import annotations

import asyncio
import functools
import inspect
import logging
import time
from typing import Any, Callable, Optional, TypeVar

R = TypeVar("R")
log = logging.getLogger(__name__)


def retry(
    max_attempts: int = 3,
    delay: float = 0.25,
    backoff_factor: float = 2.0,
    exceptions: tuple = (Exception,),
    on_retry: Optional[Callable[[Exception, int], None]] = None,
) -> Callable[[Callable[..., R]], Callable[..., R]]:
    """Call the function up to ``max_attempts`` times; after failure ``n``
    (an exception in ``exceptions``) wait ``delay * backoff_factor**(n-1)``
    seconds, call ``on_retry(exc, n)`` and try again.  The last failure is
    re-raised.  Coroutine functions are awaited and sleep with asyncio."""
    if max_attempts < 1:
        raise ValueError("max_attempts must be >= 1")

    def waits():
        d = delay
        for _ in range(max_attempts - 1):
            yield d
            d *= backoff_factor

    def decorator(func: Callable[..., R]) -> Callable[..., R]:
        if inspect.iscoroutinefunction(func):

            @functools.wraps(func)
            async def aw(*args: Any, **kwargs: Any) -> Any:
                pauses = waits()
                for attempt in range(1, max_attempts + 1):
                    try:
                        return await func(*args, **kwargs)
                    except exceptions as exc:
                        if attempt == max_attempts:
                            raise
                        if on_retry is not None:
                            on_retry(exc, attempt)
                        log.debug("retrying %s after %r (attempt %d)", func.__name__, exc, attempt)
                        await asyncio.sleep(next(pauses))
                raise AssertionError("unreachable")

            return aw  # type: ignore[return-value]

        @functools.wraps(func)
        def sw(*args: Any, **kwargs: Any) -> Any:
            pauses = waits()
            for attempt in range(1, max_attempts + 1):
                try:
                    return func(*args, **kwargs)
                except exceptions as exc:
                    if attempt == max_attempts:
                        raise
                    if on_retry is not None:
                        on_retry(exc, attempt)
                    log.debug("retrying %s after %r (attempt %d)", func.__name__, exc, attempt)
                    time.sleep(next(pauses))
            raise AssertionError("unreachable")

        return sw

    return decorator

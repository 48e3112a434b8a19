"""Concurrent rollout gathering with an exception budget.

Behaviour of the reference ``src/art/gather.py:14-257`` and
``src/art/batches.py:10-49``: ``gather_trajectory_groups`` awaits groups
concurrently under a shared :class:`GatherContext` (progress bar, running
metric means, exception budget), optionally post-processing each group;
``trajectory_group_batches`` streams fixed-size batches of finished groups.
"""

from __future__ import annotations

import asyncio
import contextlib
import contextvars
from collections import Counter
from dataclasses import dataclass, field
from typing import Any, AsyncIterator, Awaitable, Callable, Iterable, Iterator

from tqdm import auto as tqdm

from .trajectories import Trajectory, TrajectoryGroup


@dataclass
class GatherContext:
    pbar: Any = None
    metric_sums: Counter = field(default_factory=Counter)
    metric_divisors: Counter = field(default_factory=Counter)
    max_metrics: int | None = None
    max_exceptions: int | float = 0
    increment_pbar: bool = True

    def update_pbar(self, n: int) -> None:
        if self.pbar is None:
            return
        if self.increment_pbar:
            self.pbar.update(n)
        names = list(self.metric_sums.keys())
        if self.max_metrics is not None:
            names = names[: self.max_metrics]
        postfix = {
            name: self.metric_sums[name] / max(1, self.metric_divisors[name])
            for name in names
        }
        self.pbar.set_postfix(postfix)

    def too_many_exceptions(self) -> bool:
        """True once the exception count exceeds the budget.  A budget in
        (0, 1) is a fraction of the expected total; otherwise a count."""
        count = self.metric_sums["exceptions"]
        if 0 < self.max_exceptions < 1 and self.pbar is not None and self.pbar.total:
            if count / self.pbar.total <= self.max_exceptions:
                return False
        return count > self.max_exceptions

    def reset(self) -> None:
        self.pbar = None
        self.metric_sums = Counter()
        self.metric_divisors = Counter()
        self.max_exceptions = 0


_gather_context: contextvars.ContextVar[GatherContext] = contextvars.ContextVar(
    "art_b200_gather_context", default=GatherContext()
)


@contextlib.contextmanager
def set_gather_context(context: GatherContext) -> Iterator[None]:
    token = _gather_context.set(context)
    try:
        yield
    finally:
        _gather_context.reset(token)


def get_gather_context() -> GatherContext:
    return _gather_context.get()


def record_metrics(context: GatherContext, trajectory: Trajectory) -> None:
    logprobs = [
        choice.logprobs.content[0].logprob
        for choice in trajectory.messages_and_choices
        if not isinstance(choice, dict)
        and getattr(choice, "logprobs", None) is not None
        and choice.logprobs.content
    ]
    if logprobs:
        context.metric_sums["entropy"] += -sum(logprobs) / len(logprobs)
        context.metric_divisors["entropy"] += 1
    context.metric_sums["reward"] += trajectory.reward
    context.metric_divisors["reward"] += 1
    context.metric_sums.update(trajectory.metrics)
    context.metric_divisors.update(trajectory.metrics.keys())


async def wrap_group_awaitable(
    awaitable: Awaitable[TrajectoryGroup],
) -> TrajectoryGroup | None:
    context = get_gather_context()
    try:
        return await awaitable
    except Exception:
        context.metric_sums["exceptions"] += 1
        context.update_pbar(n=0)
        if context.too_many_exceptions():
            raise
        return None


async def gather_trajectory_groups(
    groups: Iterable[Awaitable[TrajectoryGroup]],
    *,
    pbar_desc: str | None = "gather",
    pbar_total_completion_tokens: bool = False,
    max_exceptions: int | float = 0,
    max_metrics: int | None = None,
    after_each: Callable[[TrajectoryGroup], Awaitable[Any]] | None = None,
) -> list[TrajectoryGroup]:
    del pbar_total_completion_tokens
    groups = list(groups)
    context = GatherContext(max_exceptions=max_exceptions, max_metrics=max_metrics)

    async def one(g: Awaitable[TrajectoryGroup]) -> Any:
        group = await wrap_group_awaitable(g)
        if group is None or after_each is None:
            return group
        return await after_each(group)

    with set_gather_context(context):
        pending = asyncio.gather(*[one(g) for g in groups])
        total = sum(getattr(g, "_num_trajectories", 1) for g in groups)
        context.pbar = tqdm.tqdm(desc=pbar_desc, total=total, disable=pbar_desc is None)
        results = await pending
    if context.pbar is not None:
        context.pbar.close()
    out: list[TrajectoryGroup] = []
    for item in results:
        if isinstance(item, list):
            out.extend(item)
        elif isinstance(item, TrajectoryGroup):
            out.append(item)
    return out


async def gather_trajectories(
    trajectories: Iterable[Awaitable[Any]],
    *,
    pbar_desc: str | None = "gather",
    pbar_total_completion_tokens: bool = False,
    max_exceptions: int | float = 0,
) -> list[Any]:
    del pbar_total_completion_tokens
    items = list(trajectories)
    context = GatherContext(max_exceptions=max_exceptions)

    async def one(awaitable: Awaitable[Any]) -> Any:
        try:
            result = await awaitable
        except BaseException as exc:
            context.metric_sums["exceptions"] += 1
            context.update_pbar(n=0)
            if context.too_many_exceptions():
                raise
            return exc
        for trajectory in result if isinstance(result, list) else [result]:
            if isinstance(trajectory, Trajectory):
                record_metrics(context, trajectory)
        context.update_pbar(n=1)
        return result

    with set_gather_context(context):
        context.pbar = tqdm.tqdm(desc=pbar_desc, total=len(items), disable=pbar_desc is None)
        results = await asyncio.gather(*[one(t) for t in items])
    context.pbar.close()
    return list(results)


async def trajectory_group_batches(
    groups: Iterable[Awaitable[TrajectoryGroup]],
    *,
    batch_size: int,
    max_batch_exceptions: int | float = 0,
    max_concurrent_batches: int = 4,
    skip_batches: int = 0,
    pbar_desc: str | None = "batches",
    pbar_total_completion_tokens: bool = False,
) -> AsyncIterator[list[TrajectoryGroup]]:
    del pbar_total_completion_tokens
    queue = list(groups)[batch_size * skip_batches :]
    pending: set[asyncio.Task] = set()
    batch: list[TrajectoryGroup] = []
    context = GatherContext(max_exceptions=max_batch_exceptions, increment_pbar=False)
    with set_gather_context(context):
        while queue or pending:
            if context.pbar is None:
                context.pbar = tqdm.tqdm(
                    desc=pbar_desc, total=batch_size, disable=pbar_desc is None
                )
            while queue and len(pending) < batch_size * max_concurrent_batches:
                pending.add(asyncio.ensure_future(wrap_group_awaitable(queue.pop(0))))
            done, pending = await asyncio.wait(pending, return_when=asyncio.FIRST_COMPLETED)
            context.pbar.update(len(done))
            batch.extend(g for task in done if (g := task.result()) is not None)
            if len(batch) >= batch_size:
                context.pbar.close()
                context.reset()
                yield batch[:batch_size]
                batch = batch[batch_size:]
        if batch:
            yield batch

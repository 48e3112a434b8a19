"""``PipelineTrainer``: rollouts, training and evaluation as three
concurrent asyncio stages.

Behaviour of the reference ``src/art/pipeline_trainer/trainer.py:70-1158``:

* ``num_rollout_workers`` workers pull scenarios, run ``rollout_fn(model,
  scenario, config) -> TrajectoryGroup`` and queue the group tagged with the
  policy version (training step) it was sampled with; a worker waits while
  the policy it would sample from is more than ``max_steps_off_policy``
  steps behind the trainer;
* the training stage takes between ``min_batch_size`` and
  ``max_batch_size`` groups, drops groups that became too stale, sets
  zero-variance groups (every reward equal: no learning signal) aside, and
  calls ``backend.train``; the KL reference lags the current step by
  ``kl_penalty_step_lag`` when given;
* the evaluation stage runs ``eval_fn(model, step, config)`` every
  ``eval_every_n_steps`` steps (and at start) and logs the result as split
  ``val``;
* checkpoints not protected (current, being evaluated, best) are pruned by a
  retention strategy; the scenario offset and step are persisted in the
  model's state so a restart resumes where it stopped;
* ``request_stop()`` (or SIGINT/SIGTERM) finishes the current step and stops.

Written from the reference's documented behaviour; the stages, the state and
the scheduling code here are this framework's own.
"""

from __future__ import annotations

import asyncio
import os
import signal
import time
from collections.abc import AsyncIterator, Awaitable, Callable, Iterable
from dataclasses import dataclass, field
from datetime import datetime, timezone
from typing import Any, Generic, TypeVar

from ..trajectories import Trajectory, TrajectoryGroup
from .checkpoint_retention import (
    CHECKPOINT_CREATED_AT_METRIC,
    CheckpointInfo,
    CheckpointRetentionContext,
    CheckpointRetentionStrategy,
)

ScenarioT = TypeVar("ScenarioT")
ConfigT = TypeVar("ConfigT")

RolloutFn = Callable[[Any, ScenarioT, ConfigT], Awaitable[TrajectoryGroup]]
SingleRolloutFn = Callable[[Any, ScenarioT, ConfigT], Awaitable[Trajectory]]
EvalFn = Callable[[Any, int, ConfigT], Awaitable[Any]]

_STATE_KEY = "pipeline_trainer"


def make_group_rollout_fn(single_rollout_fn: SingleRolloutFn, n: int) -> RolloutFn:
    """A group rollout that runs ``single_rollout_fn`` ``n`` times
    concurrently; failed rollouts are dropped from the group."""

    async def group_rollout(model: Any, scenario: Any, config: Any) -> TrajectoryGroup:
        if n <= 0:
            return TrajectoryGroup([])
        res = await asyncio.gather(*(single_rollout_fn(model, scenario, config) for _ in range(n)),
                                   return_exceptions=True)
        return TrajectoryGroup([r for r in res if isinstance(r, Trajectory)])

    return group_rollout


@dataclass
class PipelineState:
    policy_version: int = 0
    scenario_offset: int = 0
    total_scenarios_consumed: int = 0
    last_eval_step: int = -1
    discarded_stale_groups: int = 0
    zero_variance_groups: int = 0
    collapsed: bool = False  # the zero-variance failsafe stopped training
    done: bool = False
    policy_updated: asyncio.Condition = field(default_factory=asyncio.Condition)


async def _as_async_iter(src: AsyncIterator[Any] | Iterable[Any]) -> AsyncIterator[Any]:
    if hasattr(src, "__anext__"):
        async for x in src:  # type: ignore[union-attr]
            yield x
    else:
        for x in src:  # type: ignore[union-attr]
            yield x


class PipelineTrainer(Generic[ScenarioT, ConfigT]):
    def __init__(
        self,
        model: Any,
        backend: Any,
        rollout_fn: RolloutFn,
        scenarios: AsyncIterator[ScenarioT] | Iterable[ScenarioT],
        config: ConfigT,
        eval_fn: EvalFn | None = None,
        *,
        num_rollout_workers: int = 16,
        min_batch_size: int = 4,
        max_batch_size: int | None = None,
        max_steps_off_policy: int = 4,
        queue_maxsize: int | None = None,
        learning_rate: float = 1e-5,
        loss_fn: str = "cispo",
        loss_fn_config: dict | None = None,
        normalize_advantages: bool = True,
        adam_params: object | None = None,
        kl_penalty_coef: float = 0.0,
        kl_penalty_step_lag: int | None = None,
        max_steps: int | None = None,
        discard_queue_multiplier: int = 100,
        log_interval_seconds: float = 60.0,
        total_scenarios: int | None = None,
        eval_every_n_steps: int = 20,
        eval_at_start: bool = True,
        save_checkpoint: bool = True,
        checkpoint_retention_strategy: CheckpointRetentionStrategy | None = None,
        checkpoint_retention_interval: int = 1,
        resume: bool = True,
        train_kwargs: dict[str, Any] | None = None,
    ) -> None:
        checks = [
            (num_rollout_workers > 0, "num_rollout_workers must be > 0"),
            (min_batch_size > 0, "min_batch_size must be > 0"),
            (max_batch_size is None or max_batch_size >= min_batch_size, "max_batch_size must be >= min_batch_size"),
            (max_steps_off_policy >= 0, "max_steps_off_policy must be >= 0"),
            (queue_maxsize is None or queue_maxsize > 0, "queue_maxsize must be > 0"),
            (eval_every_n_steps >= 0, "eval_every_n_steps must be >= 0"),
            (max_steps is None or max_steps >= 0, "max_steps must be >= 0"),
            (log_interval_seconds > 0, "log_interval_seconds must be > 0"),
            (discard_queue_multiplier > 0, "discard_queue_multiplier must be > 0"),
            (checkpoint_retention_interval > 0, "checkpoint_retention_interval must be > 0"),
            (kl_penalty_step_lag is None or kl_penalty_step_lag >= 1, "kl_penalty_step_lag must be >= 1"),
        ]
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)
        self.model, self.backend, self.rollout_fn = model, backend, rollout_fn
        self.config, self.eval_fn = config, eval_fn
        self.num_rollout_workers = num_rollout_workers
        self.min_batch_size = min_batch_size
        self.max_batch_size = max_batch_size if max_batch_size is not None else 10 * min_batch_size
        self.max_steps_off_policy = max_steps_off_policy
        self.queue_maxsize = queue_maxsize
        self.learning_rate = learning_rate
        self.loss_fn, self.loss_fn_config = loss_fn, loss_fn_config
        self.normalize_advantages, self.adam_params = normalize_advantages, adam_params
        self.kl_penalty_coef, self.kl_penalty_step_lag = kl_penalty_coef, kl_penalty_step_lag
        self.max_steps = max_steps
        self.discard_limit = discard_queue_multiplier * min_batch_size
        self.log_interval_seconds = log_interval_seconds
        self.total_scenarios = total_scenarios
        self.eval_every_n_steps, self.eval_at_start = eval_every_n_steps, eval_at_start
        self.save_checkpoint = save_checkpoint
        self.retention = checkpoint_retention_strategy
        self.retention_interval = checkpoint_retention_interval
        self.resume = resume
        self.train_kwargs = dict(train_kwargs or {})
        self.state = PipelineState()
        self._scenarios = _as_async_iter(scenarios)
        self._scenario_lock = asyncio.Lock()
        self._discarded: list[TrajectoryGroup] = []
        self._leases: dict[int, Any] = {}  # step -> held adapter lease (scheduled evals)
        self._eval_queue: asyncio.Queue[int] | None = None
        self._output: asyncio.Queue[TrajectoryGroup | None] | None = None
        self._stop = asyncio.Event()
        self._evaluating: set[int] = set()
        self._eval_metrics: dict[int, dict[str, float]] = {}
        self.train_results: list[Any] = []

    # ------------------------------------------------------------------ control
    def request_stop(self) -> None:
        """Finish the step in progress, then stop every stage."""
        self._stop.set()

    def _persisted(self) -> dict[str, Any]:
        st = self.model.read_state() or {}
        return dict(st.get(_STATE_KEY) or {})

    def _persist(self, step: int) -> None:
        self.model.merge_state({_STATE_KEY: {
            "scenario_offset": self.state.scenario_offset, "training_step": step,
            "last_eval_step": self.state.last_eval_step,
        }})

    # ------------------------------------------------------------------ stages
    async def _next_scenario(self) -> tuple[int, Any] | None:
        async with self._scenario_lock:
            if self._stop.is_set():
                return None
            try:
                sc = await self._scenarios.__anext__()
            except StopAsyncIteration:
                return None
            off = self.state.scenario_offset
            self.state.scenario_offset += 1
            self.state.total_scenarios_consumed += 1
            return off, sc

    async def _wait_for_policy(self, version: int) -> None:
        # a worker may sample from policy `version` while the trainer has not
        # gone more than max_steps_off_policy steps past it
        cond = self.state.policy_updated
        async with cond:
            await cond.wait_for(lambda: self._stop.is_set()
                                or self._train_step_in_flight - version <= self.max_steps_off_policy)

    async def _rollout_worker(self, wid: int) -> None:
        assert self._output is not None
        while not self._stop.is_set():
            version = self.state.policy_version
            await self._wait_for_policy(version)
            nxt = await self._next_scenario()
            if nxt is None:
                return
            off, scenario = nxt
            try:
                group = await self.rollout_fn(self.model, scenario, self.config)
            except Exception as exc:  # a failed scenario does not stop the pipeline
                print(f"[pipeline] rollout worker {wid}: scenario {off} failed: {type(exc).__name__}: {exc}")
                continue
            for t in group:
                t.metadata.setdefault("policy_version", version)
                t.metadata.setdefault("scenario_offset", off)
            await self._output.put(group)

    async def _rollout_stage(self) -> None:
        assert self._output is not None
        workers = [asyncio.create_task(self._rollout_worker(i)) for i in range(self.num_rollout_workers)]
        try:
            await asyncio.gather(*workers)
        finally:
            await self._output.put(None)

    @staticmethod
    def _zero_variance(g: TrajectoryGroup) -> bool:
        rewards = [t.reward for t in g]
        return len(rewards) < 2 or max(rewards) == min(rewards)

    def _stale(self, g: TrajectoryGroup) -> bool:
        versions = [int(t.metadata.get("policy_version", self.state.policy_version)) for t in g]
        return bool(versions) and self.state.policy_version - min(versions) > self.max_steps_off_policy

    async def _collect_batch(self) -> list[TrajectoryGroup] | None:
        assert self._output is not None
        batch: list[TrajectoryGroup] = []
        finished = False
        while len(batch) < self.min_batch_size:
            g = await self._output.get()
            if g is None:
                finished = True
                break
            if self._stale(g):
                self.state.discarded_stale_groups += 1
                continue
            if self._zero_variance(g):
                self.state.zero_variance_groups += 1
                self._discarded.append(g)
                if len(self._discarded) >= self.discard_limit:
                    self._trigger_collapse()
                    return None
                continue
            batch.append(g)
        while len(batch) < self.max_batch_size and not self._output.empty():
            g = self._output.get_nowait()
            if g is None:
                finished = True
                break
            if not self._stale(g) and not self._zero_variance(g):
                batch.append(g)
        if finished:
            await self._output.put(None)  # keep the end marker for the next call
        return batch or None

    def _trigger_collapse(self) -> None:
        """Collapse failsafe (reference ``pipeline_trainer/trainer.py:879-911``):
        ``discard_queue_multiplier * min_batch_size`` zero-variance groups
        without a trainable batch in between mean the policy has collapsed to
        a degenerate output (or the reward gives no signal); training stops
        gracefully instead of spinning on useless rollouts."""
        if self.state.collapsed:
            return
        self.state.collapsed = True
        self.state.done = True
        self._stop.set()
        print(
            "\nMODEL COLLAPSE DETECTED - training stopped: "
            f"{len(self._discarded)} trajectory groups had zero reward variance "
            f"(limit {self.discard_limit} = discard_queue_multiplier {self.discard_limit // self.min_batch_size}"
            f" x min_batch_size {self.min_batch_size}).  Lower the learning rate, check that the reward "
            "varies within a group and that prompts are diverse, or raise discard_queue_multiplier.\n",
            flush=True,
        )

    def _lease_manager(self):
        get = getattr(self.backend, "adapter_leases", None)
        return get(self.model) if callable(get) else None

    async def _take_lease(self, step: int) -> None:
        """Keep checkpoint ``step`` alive (checkpoint cleanup skips leased
        steps) until :meth:`_release_lease`."""
        mgr = self._lease_manager()
        if mgr is None or step in self._leases:
            return
        cm = mgr.lease(step)
        await cm.__aenter__()
        self._leases[step] = cm

    async def _release_lease(self, step: int) -> None:
        cm = self._leases.pop(step, None)
        if cm is not None:
            await cm.__aexit__(None, None, None)

    async def _release_all_leases(self) -> None:
        for step in list(self._leases):
            await self._release_lease(step)

    async def _training_stage(self) -> None:
        while not self._stop.is_set():
            if self.max_steps is not None and self.state.policy_version >= self.max_steps:
                break
            batch = await self._collect_batch()
            if batch is None:
                break
            self._discarded.clear()
            step = self.state.policy_version
            self._train_step_in_flight = step + 1
            kwargs = dict(self.train_kwargs)
            if self.kl_penalty_coef > 0:
                kwargs["kl_penalty_coef"] = self.kl_penalty_coef
                if self.kl_penalty_step_lag is not None:
                    kwargs["kl_penalty_reference_step"] = max(0, step + 1 - self.kl_penalty_step_lag)
            versions = [int(t.metadata.get("policy_version", step)) for g in batch for t in g]
            t0 = time.monotonic()
            res = await self.backend.train(
                self.model, batch, learning_rate=self.learning_rate, loss_fn=self.loss_fn,
                loss_fn_config=self.loss_fn_config, normalize_advantages=self.normalize_advantages,
                adam_params=self.adam_params, save_checkpoint=self.save_checkpoint, **kwargs,
            )
            self.train_results.append(res)
            metrics = dict(res.metrics)
            metrics["time/step_wall_s"] = time.monotonic() - t0
            metrics["data/avg_steps_off_policy"] = sum(step - v for v in versions) / max(len(versions), 1)
            metrics["data/discarded_stale_groups"] = float(self.state.discarded_stale_groups)
            metrics["data/zero_variance_groups"] = float(self.state.zero_variance_groups)
            metrics[CHECKPOINT_CREATED_AT_METRIC] = time.time()
            await self.model.log(batch, split="train", metrics=metrics, step=res.step)
            cond = self.state.policy_updated
            async with cond:
                self.state.policy_version = res.step
                cond.notify_all()
            self._persist(res.step)
            if self._eval_queue is not None and self._should_eval(res.step):
                self._evaluating.add(res.step)
                await self._take_lease(res.step)  # released when its eval finishes
                await self._eval_queue.put(res.step)
            if res.step % self.retention_interval == 0:
                await self._prune(res.step)
        self.state.done = True
        self._stop.set()
        async with self.state.policy_updated:
            self.state.policy_updated.notify_all()

    def _should_eval(self, step: int) -> bool:
        return self.eval_fn is not None and self.eval_every_n_steps > 0 and step % self.eval_every_n_steps == 0

    async def _eval_stage(self) -> None:
        assert self._eval_queue is not None
        while True:
            step = await self._eval_queue.get()
            if step < 0:
                return
            try:
                await self._run_eval(step)
            finally:
                self._evaluating.discard(step)
                await self._release_lease(step)

    async def _run_eval(self, step: int) -> None:
        assert self.eval_fn is not None
        out = await self.eval_fn(self.model, step, self.config)
        splits = out if isinstance(out, dict) else {"val": out}
        for split, items in splits.items():
            groups = [g if isinstance(g, TrajectoryGroup) else TrajectoryGroup([g]) for g in items]
            await self.model.log(groups, split=split, step=step)
            rewards = [t.reward for g in groups for t in g]
            if rewards:
                self._eval_metrics.setdefault(step, {})[f"{split}/reward"] = sum(rewards) / len(rewards)
        self.state.last_eval_step = step

    async def _prune(self, current: int) -> None:
        if self.retention is None:
            return
        d = self.model._get_output_dir()
        ck = os.path.join(d, "checkpoints")
        if not os.path.isdir(ck):
            return
        protected = {current, *self._evaluating}
        mgr = self._lease_manager()
        if mgr is not None:
            protected |= mgr.active_steps()
        infos = []
        for name in os.listdir(ck):
            if not name.isdigit() or int(name) in protected:
                continue
            s = int(name)
            path = os.path.join(ck, name)
            infos.append(CheckpointInfo(
                step=s, path=path, created_at=datetime.fromtimestamp(os.path.getmtime(path), tz=timezone.utc),
                is_eval_step=s in self._eval_metrics, metrics=self._eval_metrics.get(s, {}),
            ))
        keep = set(self.retention(CheckpointRetentionContext(current_step=current, checkpoints=infos)))
        if any(c.step not in keep for c in infos):
            await self.backend._delete_checkpoint_files(self.model, sorted(protected | keep))

    async def _status_loop(self) -> None:
        t0 = time.monotonic()
        while not self._stop.is_set():
            try:
                await asyncio.wait_for(self._stop.wait(), timeout=self.log_interval_seconds)
            except asyncio.TimeoutError:
                pass
            total = f"/{self.total_scenarios}" if self.total_scenarios else ""
            print(f"[pipeline] step {self.state.policy_version} scenarios {self.state.scenario_offset}{total} "
                  f"stale {self.state.discarded_stale_groups} zero-var {self.state.zero_variance_groups} "
                  f"elapsed {time.monotonic() - t0:.0f}s", flush=True)

    # ------------------------------------------------------------------ entry
    async def train(self, *, handle_signals: bool = True) -> None:
        """Run the pipeline until the scenarios run out, ``max_steps`` is
        reached or a stop is requested."""
        step = await self.model.get_step()
        st = self._persisted() if self.resume else {}
        skip = int(st.get("scenario_offset", 0) or 0)
        self.state.policy_version = step
        self._train_step_in_flight = step
        self.state.last_eval_step = int(st.get("last_eval_step", -1))
        for _ in range(skip):  # resume: skip the scenarios already consumed
            try:
                await self._scenarios.__anext__()
            except StopAsyncIteration:
                break
        self.state.scenario_offset = skip
        self._output = asyncio.Queue(maxsize=self.queue_maxsize or 0)
        self._eval_queue = asyncio.Queue() if self.eval_fn is not None else None
        loop = asyncio.get_running_loop()
        installed = []
        if handle_signals:
            for sig in (signal.SIGINT, signal.SIGTERM):
                try:
                    loop.add_signal_handler(sig, self.request_stop)
                    installed.append(sig)
                except (NotImplementedError, RuntimeError, ValueError):
                    pass
        tasks = []
        try:
            if self._eval_queue is not None and self.eval_at_start and self.state.last_eval_step < step:
                await self._run_eval(step)
            eval_task = asyncio.create_task(self._eval_stage()) if self._eval_queue is not None else None
            status = asyncio.create_task(self._status_loop())
            rollout = asyncio.create_task(self._rollout_stage())
            tasks = [rollout, status] + ([eval_task] if eval_task else [])
            await self._training_stage()
            self._stop.set()
            async with self.state.policy_updated:
                self.state.policy_updated.notify_all()
            rollout.cancel()
            if eval_task is not None:
                await self._eval_queue.put(-1)
                await eval_task
            await asyncio.gather(rollout, status, return_exceptions=True)
        finally:
            for t in tasks:
                if not t.done():
                    t.cancel()
            await self._release_all_leases()
            for sig in installed:
                loop.remove_signal_handler(sig)

"""Metric taxonomy, cumulative counters, cost rollups and throughput.

Same taxonomy as the reference (``src/art/metrics.py:77-409``,
``metrics_taxonomy.py``), so dashboards built on one read the other:

* every key has a section: ``reward``, ``loss/…``, ``data/step_…``,
  ``time/step_…``, ``costs/…``, ``throughput/…``;
* ``{section}/cum/…`` is reserved: for the ``costs``, ``time`` and ``data``
  sections each flushed value is also accumulated into
  ``{section}/cum/{name without step_}`` (``data/step_trainer_tokens`` ->
  ``data/cum/trainer_tokens``);
* costs roll up: every intermediate path of a ``costs/…`` key gets the sum
  of its leaves, and ``costs/all`` the sum of the top-level children;
* a key cannot be logged both as a leaf and as an ancestor of another leaf
  in the same step;
* ``throughput/avg_trainer_tok_per_s`` = cumulative trainer tokens /
  cumulative trainer seconds (and the actor equivalent), idle times
  accumulate into ``throughput/cum/…``; ``data/cum/num_unique_scenarios``
  counts distinct scenario ids.

Builders share state per run: :meth:`MetricsBuilder.for_cost_context`
returns a builder with another cost prefix (``costs/{context}/…``) and,
optionally, its own step buffer.  The active builder is a context variable
(``activate_context`` / ``get_active``) so API-cost trackers deep in a
rollout find it.
"""

from __future__ import annotations

import asyncio
import math
import time
from contextlib import contextmanager
from contextvars import ContextVar, Token
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable

from .trajectories import TrajectoryGroup

TRAIN_GRADIENT_STEPS_KEY = "data/step_num_gradient_steps"
_CUMULATIVE_SECTIONS = ("costs", "time", "data")
_IDLE_CUM = {
    "throughput/step_trainer_idle_s": "throughput/cum/trainer_idle_s",
    "throughput/step_actor_idle_s": "throughput/cum/actor_idle_s",
}
_active: ContextVar["MetricsBuilder"] = ContextVar("art_b200_active_metrics_builder")


def is_cumulative_metric_key(key: str) -> bool:
    parts = key.split("/")
    return len(parts) >= 2 and parts[1] == "cum"


def is_builder_managed_metric(key: str) -> bool:
    return key.startswith(("costs/", "time/step_", "data/step_", "throughput/step_"))


def to_cumulative_metric_key(key: str) -> str:
    if is_cumulative_metric_key(key):
        raise ValueError(f"Metric key '{key}' is already cumulative.")
    section, rest = key.split("/", 1)
    return f"{section}/cum/{rest[5:] if rest.startswith('step_') else rest}"


def average_metric_samples(samples: Iterable[dict[str, float]]) -> dict[str, float]:
    """Key-wise mean of metric dicts; the gradient-step count must agree
    across samples and is passed through."""
    sums: dict[str, float] = {}
    counts: dict[str, int] = {}
    fixed: dict[str, float] = {}
    for s in samples:
        for k, v in s.items():
            v = float(v)
            if k == TRAIN_GRADIENT_STEPS_KEY:
                if k in fixed and fixed[k] != v:
                    raise ValueError(f"Metric '{k}' must be invariant across samples, got {fixed[k]} and {v}.")
                fixed[k] = v
            sums[k] = sums.get(k, 0.0) + v
            counts[k] = counts.get(k, 0) + 1
    return {k: fixed.get(k, sums[k] / counts[k]) for k in sums}


def _scenario_id(group: TrajectoryGroup) -> str | None:
    for md in [getattr(group, "metadata", {}) or {}] + [t.metadata or {} for t in group.trajectories]:
        for key in ("scenario_id", "scenario", "id"):
            v = md.get(key)
            if isinstance(v, (str, int)):
                return str(v)
    return None


@dataclass(frozen=True)
class TrajectoryBatchSummary:
    num_scenarios: int
    num_trajectories: int
    num_groups_submitted: int
    num_groups_trainable: int
    scenario_ids: list[str]


def _trainable(g: TrajectoryGroup) -> bool:
    rs = [t.reward for t in g.trajectories]
    return len(rs) > 1 and max(rs) != min(rs)


def summarize_trajectory_groups(groups: Iterable[TrajectoryGroup]) -> TrajectoryBatchSummary:
    groups = list(groups)
    ids: list[str] = []
    for g in groups:
        sid = _scenario_id(g)
        if sid is not None and sid not in ids:
            ids.append(sid)
    return TrajectoryBatchSummary(
        num_scenarios=len(groups),
        num_trajectories=sum(len(g.trajectories) + len(g.exceptions) for g in groups),
        num_groups_submitted=len(groups),
        num_groups_trainable=sum(1 for g in groups if _trainable(g)),
        scenario_ids=ids,
    )


def build_data_metrics_from_summary(summary: TrajectoryBatchSummary, *, include_trainable_groups: bool
                                    ) -> dict[str, float]:
    out = {
        "data/step_num_scenarios": float(summary.num_scenarios),
        "data/step_num_trajectories": float(summary.num_trajectories),
        "data/step_num_groups_submitted": float(summary.num_groups_submitted),
    }
    if include_trainable_groups:
        out["data/step_num_groups_trainable"] = float(summary.num_groups_trainable)
    return out


def summarize_groups(groups: Iterable[TrajectoryGroup]) -> dict[str, float]:
    """Reward mean / std, exceptions, trainable groups and the mean of every
    trajectory metric of a batch of groups (the per-split log line)."""
    groups = list(groups)
    rewards = [t.reward for g in groups for t in g]
    out: dict[str, float] = {
        "num_groups": float(len(groups)),
        "num_trajectories": float(len(rewards)),
        "exceptions": float(sum(len(g.exceptions) for g in groups)),
    }
    if rewards:
        mean = sum(rewards) / len(rewards)
        out["reward"] = mean
        out["reward_std_dev"] = math.sqrt(sum((r - mean) ** 2 for r in rewards) / len(rewards))
    out["num_groups_trainable"] = float(sum(1 for g in groups if _trainable(g)))
    sums: dict[str, list[float]] = {}
    for g in groups:
        for t in g:
            for k, v in t.metrics.items():
                sums.setdefault(k, []).append(float(v))
    for k, vals in sums.items():
        out[k] = sum(vals) / len(vals)
    return out


@dataclass
class _Shared:
    lock: asyncio.Lock = field(default_factory=asyncio.Lock)
    buffers: dict[str, dict[str, float]] = field(default_factory=dict)
    pending_ids: dict[str, set[str]] = field(default_factory=dict)
    cum: dict[str, float] = field(default_factory=dict)
    unique_ids: set[str] = field(default_factory=set)
    extractors: dict[str, Callable[[Any], float | None]] = field(default_factory=dict)


class MetricsBuilder:
    """Step metrics with cumulative counters, cost rollups and throughput."""

    def __init__(self, cost_context: str = "train", *, _shared: _Shared | None = None,
                 _buffer_scope: str | None = None) -> None:
        if not cost_context or not cost_context.strip():
            raise ValueError("cost_context must be non-empty")
        self.cost_context = cost_context.strip()
        self._scope = _buffer_scope if _buffer_scope is not None else self.cost_context
        self._s = _shared if _shared is not None else _Shared()
        # flat cumulative view (kept for callers that read it directly)
        self.cum = self._s.cum

    # ------------------------------------------------------------------ adding
    def _buffer(self) -> dict[str, float]:
        return self._s.buffers.setdefault(self._scope, {})

    def add_metric(self, key: str, value: float) -> None:
        if "/" not in key:
            raise ValueError("Metric key must include a section prefix")
        if is_cumulative_metric_key(key):
            raise ValueError(f"Metric key '{key}' uses the reserved cumulative namespace.")
        buf = self._buffer()
        for other in buf:
            if other != key and other.startswith(key + "/"):
                raise ValueError(f"Cannot log '{key}' as a leaf: it is an ancestor of '{other}'.")
            if other != key and key.startswith(other + "/"):
                raise ValueError(f"Cannot log '{key}' as a leaf: '{other}' is already a leaf ancestor.")
        buf[key] = buf.get(key, 0.0) + float(value)

    def add_cost(self, path: str, usd: float) -> None:
        if not path:
            raise ValueError("Cost path must be non-empty")
        self.add_metric(f"costs/{path}", usd)

    def add_response_cost(self, source: str, response: Any, *, provider: str, model_name: str,
                          prompt_price_per_million: float | None = None,
                          completion_price_per_million: float | None = None,
                          cached_prompt_price_per_million: float | None = None) -> float | None:
        """Price one API response (``usage`` token counts) under
        ``costs/{cost_context}/{source}``; explicit prices win over registered
        ones, a registered provider extractor over both."""
        from .costs import TokenPricing, api_call_cost, register_api_pricing

        src = source.strip("/")
        if not src:
            raise ValueError("source must be non-empty")
        ext = self._s.extractors.get(provider.strip().lower())
        if ext is not None:
            cost = ext(response)
        else:
            if prompt_price_per_million is not None and completion_price_per_million is not None:
                register_api_pricing(model_name, TokenPricing(prompt_price_per_million, completion_price_per_million,
                                                              cached_prompt_price_per_million))
            cost = api_call_cost(response, model_name)
        if cost is None:
            return None
        self.add_cost(f"{self.cost_context}/{src}", cost)
        return cost

    def register_cost_extractor(self, provider: str, extractor: Callable[[Any], float | None]) -> None:
        p = provider.strip().lower()
        if not p:
            raise ValueError("provider must be non-empty")
        self._s.extractors[p] = extractor

    def register_model_pricing(self, model_name: str, *, prompt_per_million: float, completion_per_million: float,
                               cached_prompt_per_million: float | None = None) -> None:
        from .costs import TokenPricing, register_api_pricing

        if not model_name.strip():
            raise ValueError("model_name must be non-empty")
        register_api_pricing(model_name, TokenPricing(prompt_per_million, completion_per_million,
                                                      cached_prompt_per_million))

    def add_data(self, step_num_scenarios: int | None = None, step_actor_tokens: int | None = None,
                 scenario_ids: list[str] | None = None) -> None:
        if step_num_scenarios is not None:
            self.add_metric("data/step_num_scenarios", step_num_scenarios)
        if step_actor_tokens is not None:
            self.add_metric("data/step_actor_tokens", step_actor_tokens)
        if scenario_ids is not None:
            self._s.pending_ids.setdefault(self._scope, set()).update(str(x) for x in scenario_ids)

    def add_user_timing(self, step_wall_s: float | None = None, step_actor_s: float | None = None,
                        step_eval_s: float | None = None) -> None:
        for name, v in (("time/step_wall_s", step_wall_s), ("time/step_actor_s", step_actor_s),
                        ("time/step_eval_s", step_eval_s)):
            if v is not None:
                self.add_metric(name, v)

    def add_idle_times(self, step_trainer_idle_s: float | None = None, step_actor_idle_s: float | None = None) -> None:
        if step_trainer_idle_s is not None:
            self.add_metric("throughput/step_trainer_idle_s", step_trainer_idle_s)
        if step_actor_idle_s is not None:
            self.add_metric("throughput/step_actor_idle_s", step_actor_idle_s)

    @contextmanager
    def measure(self, key: str):
        t0 = time.monotonic()
        try:
            yield
        finally:
            self.add_metric(key, time.monotonic() - t0)

    # ------------------------------------------------------------------ flushing
    @staticmethod
    def _rollups(costs: dict[str, float]) -> dict[str, float]:
        if not costs:
            return {}
        out: dict[str, float] = {}
        for key in costs:
            parts = key.split("/")
            for d in range(2, len(parts)):
                parent = "/".join(parts[:d])
                if parent not in out:
                    out[parent] = sum(v for k, v in costs.items() if k.startswith(parent + "/"))
        tops = {k.split("/")[1] for k in costs}
        out["costs/all"] = sum(out.get(f"costs/{t}", costs.get(f"costs/{t}", 0.0)) for t in tops)
        return out

    def _finish(self, result: dict[str, float], ids: set[str]) -> dict[str, float]:
        result.update(self._rollups({k: v for k, v in result.items() if k.startswith("costs/")}))
        for key, v in list(result.items()):
            if key.split("/", 1)[0] in _CUMULATIVE_SECTIONS and not is_cumulative_metric_key(key):
                ck = to_cumulative_metric_key(key)
                self._s.cum[ck] = self._s.cum.get(ck, 0.0) + v
                result[ck] = self._s.cum[ck]
        if ids:
            self._s.unique_ids.update(ids)
            result["data/cum/num_unique_scenarios"] = float(len(self._s.unique_ids))
        for step_key, cum_key in _IDLE_CUM.items():
            if step_key in result:
                self._s.cum[cum_key] = self._s.cum.get(cum_key, 0.0) + result[step_key]
                result[cum_key] = self._s.cum[cum_key]
        for who in ("trainer", "actor"):
            tok, sec = self._s.cum.get(f"data/cum/{who}_tokens"), self._s.cum.get(f"time/cum/{who}_s")
            if (f"data/step_{who}_tokens" in result or f"time/step_{who}_s" in result) and tok and sec:
                result[f"throughput/avg_{who}_tok_per_s"] = tok / sec
        step_tok, step_sec = result.get("data/step_trainer_tokens"), result.get("time/step_trainer_s")
        if step_tok is not None and step_sec:
            result["throughput/step_trainer_tok_per_s"] = step_tok / step_sec
        return result

    async def flush(self) -> dict[str, float]:
        """The step's metrics plus rollups and cumulative values; clears the
        step buffer of this builder's scope."""
        async with self._s.lock:
            return self.flush_sync()

    def flush_sync(self) -> dict[str, float]:
        result = dict(self._buffer())
        ids = set(self._s.pending_ids.get(self._scope, set()))
        self._buffer().clear()
        self._s.pending_ids.pop(self._scope, None)
        return self._finish(result, ids)

    def update(self, step_metrics: dict[str, float]) -> dict[str, float]:
        """One training step's metrics (already summed by the trainer) with
        the cumulative counters and throughput added."""
        buf = {k: float(v) for k, v in step_metrics.items()}
        return self._finish(buf, set())

    # ------------------------------------------------------------------ scopes / state
    def for_cost_context(self, cost_context: str, *, buffer_scope: str | None = None) -> "MetricsBuilder":
        cc = cost_context.strip()
        if not cc:
            raise ValueError("cost_context must be non-empty")
        scope = buffer_scope.strip() if buffer_scope is not None else cc
        if not scope:
            raise ValueError("buffer_scope must be non-empty")
        if cc == self.cost_context and scope == self._scope:
            return self
        return MetricsBuilder(cc, _shared=self._s, _buffer_scope=scope)

    def activate(self) -> Token:
        return _active.set(self)

    @contextmanager
    def activate_context(self):
        tok = self.activate()
        try:
            yield self
        finally:
            _active.reset(tok)

    @staticmethod
    def get_active() -> "MetricsBuilder":
        return _active.get()

    def state_dict(self) -> dict[str, Any]:
        return {"cum_state": dict(self._s.cum), "unique_scenario_ids": sorted(self._s.unique_ids)}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self._s.cum.clear()
        self._s.cum.update({str(k): float(v) for k, v in (state.get("cum_state") or {}).items()})
        self._s.unique_ids.clear()
        self._s.unique_ids.update(str(x) for x in state.get("unique_scenario_ids") or [])
        self._s.buffers.clear()
        self._s.pending_ids.clear()

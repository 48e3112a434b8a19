"""Cost accounting: training / sampling token prices, GPU time, and API
(judge) calls.

Same role as the reference ``src/art/costs.py:10-158`` and
``api_costs.py`` (``track_api_cost``): per-model token prices turn token
counts into dollars, reported as ``costs/...`` metrics; API responses
(OpenAI-style ``usage``) are priced per call and accumulated under a
``judge/...`` or other source name.  Prices are configuration, not shipped
data: register them with :func:`register_model_pricing` /
:func:`register_api_pricing` (or pass a GPU-hour price), since they change
with the provider.
"""

from __future__ import annotations

import functools
import threading
from dataclasses import dataclass
from typing import Any, Callable


@dataclass(frozen=True)
class ModelPricing:
    """Dollars per million tokens."""

    prefill: float
    sample: float
    train: float


@dataclass(frozen=True)
class TokenPricing:
    """API prices, dollars per million tokens."""

    prompt: float
    completion: float
    cached_prompt: float | None = None


MODEL_PRICING: dict[str, ModelPricing] = {}
API_PRICING: dict[str, TokenPricing] = {}


def register_model_pricing(model: str, pricing: ModelPricing) -> None:
    MODEL_PRICING[model] = pricing


def register_api_pricing(model: str, pricing: TokenPricing) -> None:
    API_PRICING[_normalize(model)] = pricing


def _normalize(model: str) -> str:
    return model.split("/", 1)[1] if "/" in model else model


def get_model_pricing(model: str) -> ModelPricing | None:
    return MODEL_PRICING.get(model) or MODEL_PRICING.get(_normalize(model))


def compute_train_cost(model: str, trainer_tokens: float | None, prefill_tokens: float | None = None,
                       sample_tokens: float | None = None) -> dict[str, float]:
    """``costs/train``, ``costs/prefill``, ``costs/sample`` for one step
    (empty when the model has no registered price)."""
    p = get_model_pricing(model)
    if p is None:
        return {}
    out = {}
    if trainer_tokens:
        out["costs/train"] = trainer_tokens * p.train / 1e6
    if prefill_tokens:
        out["costs/prefill"] = prefill_tokens * p.prefill / 1e6
    if sample_tokens:
        out["costs/sample"] = sample_tokens * p.sample / 1e6
    return out


def gpu_time_cost(seconds: float, gpus: int, usd_per_gpu_hour: float) -> dict[str, float]:
    return {"costs/gpu": seconds / 3600.0 * gpus * usd_per_gpu_hour}


def _usage_counts(response: Any) -> tuple[float, float, float]:
    usage = getattr(response, "usage", None)
    if usage is None and isinstance(response, dict):
        usage = response.get("usage")
    if usage is None:
        return 0.0, 0.0, 0.0

    def read(obj: Any, *path: str) -> float:
        for k in path:
            obj = obj.get(k) if isinstance(obj, dict) else getattr(obj, k, None)
            if obj is None:
                return 0.0
        return float(obj)

    prompt = read(usage, "prompt_tokens") or read(usage, "input_tokens")
    completion = read(usage, "completion_tokens") or read(usage, "output_tokens")
    cached = read(usage, "prompt_tokens_details", "cached_tokens")
    return prompt, completion, cached


def api_call_cost(response: Any, model: str) -> float | None:
    """Dollars for one API response (``None`` without a registered price)."""
    p = API_PRICING.get(_normalize(model))
    if p is None:
        return None
    prompt, completion, cached = _usage_counts(response)
    cached_rate = p.cached_prompt if p.cached_prompt is not None else p.prompt
    return ((prompt - cached) * p.prompt + cached * cached_rate + completion * p.completion) / 1e6


class CostTracker:
    """Thread-safe accumulator of ``costs/{source}`` values."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self.totals: dict[str, float] = {}

    def add(self, source: str, dollars: float) -> None:
        with self._lock:
            key = f"costs/{source}"
            self.totals[key] = self.totals.get(key, 0.0) + dollars

    def drain(self) -> dict[str, float]:
        with self._lock:
            out, self.totals = self.totals, {}
            return out


DEFAULT_TRACKER = CostTracker()


def track_api_cost(source: str, model: str, tracker: CostTracker | None = None):
    """Decorator for async functions returning an API response: each call's
    cost is added to ``costs/{source}``."""
    tr = tracker or DEFAULT_TRACKER

    def deco(fn: Callable[..., Any]):
        @functools.wraps(fn)
        async def wrapper(*args: Any, **kwargs: Any):
            resp = await fn(*args, **kwargs)
            c = api_call_cost(resp, kwargs.get("model", model))
            if c is not None:
                tr.add(source, c)
            return resp

        return wrapper

    return deco

import asyncio
from types import SimpleNamespace

from art_mlx_b200.costs import (
    CostTracker,
    ModelPricing,
    TokenPricing,
    api_call_cost,
    compute_train_cost,
    register_api_pricing,
    register_model_pricing,
    track_api_cost,
)


def test_costs():
    register_model_pricing("my/model", ModelPricing(prefill=1.0, sample=2.0, train=3.0))
    c = compute_train_cost("my/model", 2e6, 1e6, 0)
    assert c == {"costs/train": 6.0, "costs/prefill": 1.0}
    assert compute_train_cost("unknown", 10) == {}
    register_api_pricing("openai/judge", TokenPricing(prompt=1.0, completion=4.0, cached_prompt=0.5))
    resp = SimpleNamespace(usage=SimpleNamespace(prompt_tokens=1000, completion_tokens=500,
                                                 prompt_tokens_details=SimpleNamespace(cached_tokens=200)))
    assert abs(api_call_cost(resp, "judge") - (800 * 1 + 200 * 0.5 + 500 * 4) / 1e6) < 1e-12
    tr = CostTracker()

    @track_api_cost("judge/ruler", "judge", tracker=tr)
    async def call():
        return resp

    asyncio.run(call())
    asyncio.run(call())
    assert abs(tr.drain()["costs/judge/ruler"] - 2 * 0.0029) < 1e-9

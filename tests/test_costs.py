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


def test_metrics_taxonomy_rollups_cumulative_and_throughput():
    import asyncio

    import pytest

    from art_mlx_b200.metrics import MetricsBuilder, average_metric_samples, to_cumulative_metric_key

    b = MetricsBuilder("train")
    judge = b.for_cost_context("eval")
    b.add_cost("train/gpu", 1.5)
    b.add_cost("train/judge/gpt", 0.25)
    judge.add_cost("eval/judge", 0.5)  # own buffer scope
    b.add_metric("data/step_trainer_tokens", 1000)
    b.add_metric("time/step_trainer_s", 2.0)
    b.add_data(step_num_scenarios=3, scenario_ids=["a", "b"])
    b.add_idle_times(step_trainer_idle_s=0.5)
    with pytest.raises(ValueError):
        b.add_metric("costs/train/gpu/extra", 1.0)  # gpu is already a leaf
    with pytest.raises(ValueError):
        b.add_metric("data/cum/x", 1.0)  # reserved namespace
    with pytest.raises(ValueError):
        b.add_metric("nosection", 1.0)
    m = asyncio.run(b.flush())
    assert m["costs/train"] == 1.75 and m["costs/train/judge"] == 0.25 and m["costs/all"] == 1.75
    assert m["costs/cum/train/gpu"] == 1.5 and m["data/cum/trainer_tokens"] == 1000
    assert m["throughput/avg_trainer_tok_per_s"] == 500 and m["throughput/cum/trainer_idle_s"] == 0.5
    assert m["data/cum/num_unique_scenarios"] == 2
    j = asyncio.run(judge.flush())
    assert j["costs/all"] == 0.5 and j["costs/cum/eval/judge"] == 0.5
    b.add_metric("data/step_trainer_tokens", 500)
    b.add_metric("time/step_trainer_s", 3.0)
    b.add_data(scenario_ids=["b", "c"])
    m2 = asyncio.run(b.flush())
    assert m2["data/cum/trainer_tokens"] == 1500 and m2["throughput/avg_trainer_tok_per_s"] == 300
    assert m2["data/cum/num_unique_scenarios"] == 3
    state = b.state_dict()
    fresh = MetricsBuilder("train")
    fresh.load_state_dict(state)
    fresh.add_metric("data/step_trainer_tokens", 100)
    assert asyncio.run(fresh.flush())["data/cum/trainer_tokens"] == 1600
    assert to_cumulative_metric_key("time/step_wall_s") == "time/cum/wall_s"
    with pytest.raises(ValueError):
        average_metric_samples([{"data/step_num_gradient_steps": 1}, {"data/step_num_gradient_steps": 2}])
    assert average_metric_samples([{"loss/train": 1.0}, {"loss/train": 3.0}]) == {"loss/train": 2.0}
    with b.activate_context():
        assert MetricsBuilder.get_active() is b

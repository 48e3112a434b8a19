"""PipelineTrainer on CPU: rollout workers, batched training through
LocalBackend, evaluation, zero-variance filtering, resume, retention."""

import asyncio
import os
import random

import pytest

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.pipeline_trainer import PipelineTrainer, keep_recent_and_top, make_group_rollout_fn
from art_mlx_b200.preprocessing.synthetic import make_choice
from art_mlx_b200.trajectories import Trajectory


def _model():
    return art.TrainableModel(name="pipe", project="p", base_model="tiny-qwen3",
                              _internal_config={"peft_args": {"r": 4, "lora_alpha": 8}})


async def _single(model, scenario, config):
    rng = random.Random()
    await asyncio.sleep(0.001)
    prompt = scenario["prompt"]
    comp = [rng.randrange(1024) for _ in range(8)]
    reward = 1.0 if scenario.get("constant") else rng.random()
    return Trajectory(messages_and_choices=[{"role": "user", "content": "s"},
                                            make_choice(prompt, comp, [-1.0] * 8)], reward=reward)


def _scenarios(n, start=0):
    rng = random.Random(1)
    out = []
    for i in range(n):
        out.append({"prompt": [rng.randrange(1024) for _ in range(16)], "constant": i % 5 == 4, "i": start + i})
    return out


async def _eval(model, step, config):
    return [Trajectory(messages_and_choices=[{"role": "user", "content": "e"}], reward=float(step))]


def test_pipeline_trains_evaluates_and_resumes(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        pt = PipelineTrainer(model, backend, make_group_rollout_fn(_single, 4), _scenarios(20), config=None,
                             eval_fn=_eval, num_rollout_workers=3, min_batch_size=2, max_batch_size=2,
                             max_steps=3, eval_every_n_steps=2, learning_rate=1e-4, log_interval_seconds=30,
                             checkpoint_retention_strategy=keep_recent_and_top(recent=1, top=1))
        await pt.train(handle_signals=False)
        assert await model.get_step() == 3
        assert len(pt.train_results) == 3
        assert pt.state.zero_variance_groups >= 1  # every 5th scenario has constant rewards
        hist = open(os.path.join(model._get_output_dir(), "history.jsonl")).read()
        assert '"val/reward"' in hist and '"train/' in hist
        # retention kept the current step and at most one more
        ck = sorted(int(d) for d in os.listdir(os.path.join(model._get_output_dir(), "checkpoints")))
        assert ck[-1] == 3 and len(ck) <= 3
        consumed = pt.state.scenario_offset
        # resume: a new pipeline continues from the persisted scenario offset
        pt2 = PipelineTrainer(model, backend, make_group_rollout_fn(_single, 4), _scenarios(20), config=None,
                              num_rollout_workers=2, min_batch_size=2, max_steps=4, learning_rate=1e-4)
        await pt2.train(handle_signals=False)
        assert await model.get_step() == 4
        assert pt2.state.scenario_offset > consumed

    asyncio.run(go())


def test_pipeline_validates_arguments(tmp_path):
    with pytest.raises(ValueError, match="min_batch_size"):
        PipelineTrainer(None, None, None, [], None, min_batch_size=0)
    with pytest.raises(ValueError, match="max_batch_size"):
        PipelineTrainer(None, None, None, [], None, min_batch_size=4, max_batch_size=2)


def test_collapse_failsafe_stops_training_gracefully(tmp_path):
    """Every group has constant rewards: after discard_queue_multiplier x
    min_batch_size of them the trainer stops (no exception, no step)."""
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        scen = [dict(s, constant=True) for s in _scenarios(40)]
        pt = PipelineTrainer(model, backend, make_group_rollout_fn(_single, 2), scen, config=None,
                             num_rollout_workers=2, min_batch_size=2, max_batch_size=2, max_steps=3,
                             discard_queue_multiplier=3, learning_rate=1e-4, log_interval_seconds=30)
        await pt.train(handle_signals=False)
        assert pt.state.collapsed and pt.state.done
        assert pt.state.zero_variance_groups >= 6
        assert await model.get_step() == 0 and not pt.train_results

    asyncio.run(go())


def test_scheduled_eval_holds_an_adapter_lease(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        seen = []

        async def slow_eval(m, step, config):
            seen.append((step, step in backend.adapter_leases(m).active_steps()))
            return [Trajectory(messages_and_choices=[{"role": "user", "content": "e"}], reward=1.0)]

        pt = PipelineTrainer(model, backend, make_group_rollout_fn(_single, 4), _scenarios(20), config=None,
                             eval_fn=slow_eval, num_rollout_workers=2, min_batch_size=2, max_batch_size=2,
                             max_steps=2, eval_every_n_steps=1, learning_rate=1e-4, log_interval_seconds=30)
        await pt.train(handle_signals=False)
        # evals scheduled after a training step run on a leased checkpoint (the
        # start-of-run eval runs before training, synchronously)
        assert seen and all(held for step, held in seen if step > 0) and any(step > 0 for step, _ in seen)
        assert not backend.adapter_leases(model).active_steps()  # and released afterwards

    asyncio.run(go())

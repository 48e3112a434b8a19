"""Streaming helpers, auto-recorded and yielded trajectories, against the
native rollout server on CPU."""

import asyncio
import socket

import art_mlx_b200 as art
from art_mlx_b200.auto_trajectory import auto_trajectory, capture_auto_trajectory
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.openai import consume_chat_completion_stream
from art_mlx_b200.yield_trajectory import capture_yielded_trajectory, yield_trajectory


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_auto_trajectory_records_calls_and_streams(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu", inference="native")
        model = art.TrainableModel(name="auto", project="p", base_model="tiny-qwen3",
                                   _internal_config={"peft_args": {"r": 4, "lora_alpha": 8}})
        try:
            await model.register(backend, _openai_client_config={"port": _port()})
            client = model.openai_client()
            name = model.get_inference_name()

            async def agent():
                msgs = [{"role": "user", "content": "hi"}]
                r1 = await client.chat.completions.create(model=name, messages=msgs, max_tokens=4)
                msgs += [{"role": "assistant", "content": r1.choices[0].message.content}, {"role": "user", "content": "more"}]
                stream = await client.chat.completions.create(model=name, messages=msgs, max_tokens=4, stream=True)
                r2 = await consume_chat_completion_stream(stream)
                assert r2.choices[0].message.content == r2.choices[0].message.content
                # an unrelated side conversation goes to an additional history
                await client.chat.completions.create(model=name, messages=[{"role": "user", "content": "judge"}],
                                                     max_tokens=2)
                auto_trajectory(required=True).reward = 1.5

            t = await capture_auto_trajectory(agent())
            assert t.reward == 1.5
            mc = t.messages_and_choices
            assert len(mc) == 4  # user, choice, user, choice (the assistant turn is the recorded choice)
            from openai.types.chat.chat_completion import Choice

            assert isinstance(mc[1], Choice) and isinstance(mc[3], Choice)
            assert mc[3].model_extra.get("token_ids") and mc[3].model_extra.get("prompt_token_ids")
            assert len(t.additional_histories) == 1
            # recorded trajectories train directly
            res = await backend.train(model, [art.TrajectoryGroup([t, t.model_copy(update={"reward": 0.0})])],
                                      learning_rate=1e-4)
            assert res.step == 1 and res.metrics["data/step_trainer_tokens"] > 0

            async def yielding():
                yield_trajectory(art.Trajectory(messages_and_choices=[], reward=2.0))
                return "done"

            y = await capture_yielded_trajectory(yielding())
            assert y.reward == 2.0
        finally:
            await backend.close()

    asyncio.run(go())

"""The whole RL loop on CPU through the public API: the native rollout
server samples from the live policy over HTTP (OpenAI client), trajectories
carry the server's token ids, LocalBackend trains on them, and the next
rollouts come from the updated adapter."""

import asyncio
import socket

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rollout_train_rollout_loop(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu", inference="native")
        model = art.TrainableModel(name="loop", project="p", base_model="tiny-qwen3",
                                   _internal_config={"peft_args": {"r": 4, "lora_alpha": 8}})
        try:
            await model.register(backend, _openai_client_config={"port": _port()})
            client = model.openai_client()
            names = [m.id for m in (await client.models.list()).data]
            assert "loop" in names

            async def rollout(seed):
                resp = await client.chat.completions.create(
                    model=model.get_inference_name(), messages=[{"role": "user", "content": f"say {seed}"}],
                    n=4, max_tokens=6, temperature=1.0, seed=seed, logprobs=True,
                )
                trajs = []
                for i, ch in enumerate(resp.choices):
                    assert ch.model_extra["token_ids"] and ch.model_extra["prompt_token_ids"]
                    assert len(ch.logprobs.content) == len(ch.model_extra["token_ids"])
                    trajs.append(art.Trajectory(messages_and_choices=[{"role": "user", "content": f"say {seed}"}, ch],
                                                reward=float(i)))
                return art.TrajectoryGroup(trajs)

            groups = await asyncio.gather(*(rollout(s) for s in range(3)))
            res = await backend.train(model, groups, learning_rate=1e-3)
            assert res.step == 1 and res.metrics["data/step_trainer_tokens"] > 0
            assert model.get_inference_name() == "loop@1"
            # the new policy serves immediately; the old step stays addressable
            again = await rollout(7)
            assert len(again.trajectories) == 4
            old = await client.chat.completions.create(model="loop@0", messages=[{"role": "user", "content": "x"}],
                                                       max_tokens=3, temperature=0.0)
            assert old.choices[0].model_extra["token_ids"]
            # in-process entry point (no HTTP)
            out = await backend.create_chat_completion(model, [{"role": "user", "content": "hi"}], max_tokens=3)
            assert out["choices"][0]["token_ids"] and out["prompt_token_ids"]
        finally:
            await backend.close()

    asyncio.run(go())

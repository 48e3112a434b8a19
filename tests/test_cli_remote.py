"""CLI commands (init, migrate) and the RemoteBackend against an in-process
``run`` server."""

import asyncio
import json
import os
import socket
import threading
import time

import pyarrow.parquet as pq

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.backends.remote import RemoteBackend
from art_mlx_b200.cli import build_server_app, main
from art_mlx_b200.preprocessing.synthetic import synthetic_groups


def test_init_and_migrate(tmp_path):
    assert main(["init", str(tmp_path / "proj")]) == 0
    assert (tmp_path / "proj" / "train.py").exists()
    d = tmp_path / "m" / "trajectories" / "train"
    d.mkdir(parents=True)
    group = {"trajectories": [
        {"messages_and_choices": [{"role": "user", "content": "hi"},
                                  {"finish_reason": "stop", "index": 0,
                                   "message": {"role": "assistant", "content": "yo"}}], "reward": 1.5},
        {"messages_and_choices": [{"role": "user", "content": "hi"}], "reward": 0.5},
    ]}
    (d / "0001.jsonl").write_text(json.dumps(group) + "\n")
    (tmp_path / "m" / "history.jsonl").write_text('{"step": 1}\n')
    assert main(["migrate", str(tmp_path / "m")]) == 0
    assert not (d / "0001.jsonl").exists() and (tmp_path / "m" / "history.jsonl").exists()
    rows = pq.read_table(d / "0001.parquet").to_pylist()
    assert [r["reward"] for r in rows] == [1.5, 0.5]
    assert json.loads(rows[0]["messages"])[1]["content"] == "yo"


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_remote_backend_trains_through_http(tmp_path):
    import uvicorn

    port = _port()
    server = uvicorn.Server(uvicorn.Config(build_server_app(LocalBackend(path=str(tmp_path), device="cpu")),
                                           host="127.0.0.1", port=port, log_level="warning"))
    t = threading.Thread(target=server.run, daemon=True)
    t.start()
    while not server.started:
        time.sleep(0.01)

    async def go():
        backend = RemoteBackend(f"http://127.0.0.1:{port}")
        assert await backend.healthcheck()
        model = art.TrainableModel(name="remote", project="p", base_model="tiny-qwen3",
                                   _internal_config={"peft_args": {"r": 4, "lora_alpha": 8}})
        await model.register(backend)
        assert await model.get_step() == 0
        groups = synthetic_groups(num_groups=2, rollouts_per_group=4, prompt_len=16, completion_len=8,
                                  vocab_size=1024, seed=0)
        res = await backend.train(model, groups, learning_rate=1e-4)
        assert res.step == 1 and res.metrics["data/step_trainer_tokens"] == 2 * 4 * 8
        assert os.path.exists(os.path.join(res.checkpoint_path, "adapter_model.safetensors"))
        assert model.get_inference_name() == "remote@1"
        await backend.close()

    try:
        asyncio.run(go())
    finally:
        server.should_exit = True
        t.join(10)

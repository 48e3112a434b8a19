"""The vLLM runtime manager: server command, start (health + model list),
adapter hot-load / reload / unload and shutdown, against a stand-in server
process (the real vLLM server runs in tests/test_vllm_runtime_gpu.py)."""

import asyncio
import os
import sys

import httpx

from art_mlx_b200.runtime.vllm_runtime import ManagedVllmRuntime, VllmRuntimeConfig, build_server_cmd

HERE = os.path.dirname(os.path.abspath(__file__))


def test_server_command():
    cmd = build_server_cmd(VllmRuntimeConfig(base_model="/m", served_model_name="agent", port=1234, max_lora_rank=16,
                                             api_key="k", skip_tokenizer=True,
                                             engine_args={"enforce_eager": True, "max_model_len": 512}))
    assert cmd[1:3] == ["-m", "vllm.entrypoints.openai.api_server"]
    for a in ("--enable-lora", "--skip-tokenizer-init", "--enforce-eager"):
        assert a in cmd
    assert cmd[cmd.index("--max-lora-rank") + 1] == "16" and cmd[cmd.index("--max-model-len") + 1] == "512"


def test_runtime_lifecycle_and_hot_load(tmp_path):
    cfg = VllmRuntimeConfig(base_model="/m", served_model_name="agent",
                            server_cmd=[sys.executable, os.path.join(HERE, "fake_vllm_server.py"), "{host}", "{port}"])
    rt = ManagedVllmRuntime(cfg, log_path=str(tmp_path / "vllm.log"))

    async def go():
        url = await rt.start(timeout_s=60)
        assert url.endswith("/v1")
        await rt.load_lora("agent@1", str(tmp_path / "ck1"))
        await rt.load_lora("agent@1", str(tmp_path / "ck1b"))  # reload: unload then load
        await rt.load_lora("agent@2", str(tmp_path / "ck2"))
        async with httpx.AsyncClient() as c:
            ids = {m["id"]: m.get("root") for m in (await c.get(url + "/models")).json()["data"]}
        assert ids["agent@1"].endswith("ck1b") and "agent@2" in ids
        await rt.unload_lora("agent@2")
        assert rt.loaded == {"agent@1"}

    try:
        asyncio.run(go())
        proc = rt.process
    finally:
        rt.close()
    assert proc.poll() is not None and rt.process is None

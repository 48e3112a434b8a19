"""A vLLM OpenAI server as the rollout engine, with LoRA adapters hot-loaded.

Role of the reference ``src/art/vllm_runtime.py`` (``ManagedVllmRuntime``,
``build_vllm_runtime_server_cmd``, ``wait_for_vllm_runtime``) and of its
LoRA hot-load in ``src/art/unsloth/service.py:628-767``: the trainer publishes
a PEFT checkpoint per step and the server serves it as ``{name}@{step}``
without a restart.  The server is vLLM's own ``openai.api_server`` (the
package in this image), started as a managed child process (own session,
parent-death signal: it never outlives the trainer) on the GPUs named by
``gpus`` (dedicated mode: the trainer keeps its own GPUs).  Adapters move by
path (``/v1/load_lora_adapter``); with ``skip_tokenizer`` the server takes
token-id prompts, which is what a trainer that never re-tokenizes sends.
"""

from __future__ import annotations

import asyncio
import os
import subprocess
import sys
import time
from dataclasses import dataclass, field
from typing import Any

from ..utils import managed_process


@dataclass
class VllmRuntimeConfig:
    base_model: str
    served_model_name: str
    host: str = "127.0.0.1"
    port: int = 0  # 0: a free port
    gpus: str | None = None  # CUDA_VISIBLE_DEVICES of the server (None: inherit)
    max_lora_rank: int = 64
    max_loras: int = 4
    api_key: str | None = None
    skip_tokenizer: bool = False
    engine_args: dict[str, Any] = field(default_factory=dict)  # extra --flag value pairs
    server_cmd: list[str] | None = None  # replaces the vLLM command (tests run a stand-in server)


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def build_server_cmd(cfg: VllmRuntimeConfig) -> list[str]:
    if cfg.server_cmd is not None:
        return [c.format(host=cfg.host, port=cfg.port) for c in cfg.server_cmd]
    cmd = [sys.executable, "-m", "vllm.entrypoints.openai.api_server", "--model", cfg.base_model,
           "--served-model-name", cfg.served_model_name, "--host", cfg.host, "--port", str(cfg.port),
           "--enable-lora", "--max-lora-rank", str(cfg.max_lora_rank), "--max-loras", str(cfg.max_loras)]
    if cfg.api_key:
        cmd += ["--api-key", cfg.api_key]
    if cfg.skip_tokenizer:
        cmd += ["--skip-tokenizer-init"]
    for k, v in cfg.engine_args.items():
        flag = "--" + k.replace("_", "-")
        if v is True:
            cmd.append(flag)
        elif v is not False and v is not None:
            cmd += [flag, str(v)]
    return cmd


class ManagedVllmRuntime:
    def __init__(self, cfg: VllmRuntimeConfig, log_path: str | None = None) -> None:
        self.cfg = cfg
        self.log_path = log_path
        self.process: subprocess.Popen | None = None
        self._log = None
        self.loaded: set[str] = set()

    @property
    def base_url(self) -> str:
        return f"http://{self.cfg.host}:{self.cfg.port}"

    def headers(self) -> dict[str, str]:
        return {"Authorization": f"Bearer {self.cfg.api_key}"} if self.cfg.api_key else {}

    async def start(self, timeout_s: float = 900.0) -> str:
        """Launch the server and wait until ``/health`` answers and the base
        model is listed; returns the OpenAI base URL."""
        import httpx

        if not self.cfg.port:
            self.cfg.port = _free_port()
        env = dict(os.environ)
        env["VLLM_ALLOW_RUNTIME_LORA_UPDATING"] = "True"
        if self.cfg.gpus is not None:
            env["CUDA_VISIBLE_DEVICES"] = self.cfg.gpus
        out = subprocess.DEVNULL
        if self.log_path:
            os.makedirs(os.path.dirname(self.log_path) or ".", exist_ok=True)
            self._log = open(self.log_path, "w", buffering=1)
            out = self._log
        self.process = managed_process.popen(build_server_cmd(self.cfg), stdout=out, stderr=subprocess.STDOUT, env=env)
        deadline = time.monotonic() + timeout_s
        async with httpx.AsyncClient() as client:
            while True:
                if self.process.poll() is not None:
                    raise RuntimeError(f"vLLM server exited with code {self.process.returncode} (log: {self.log_path})")
                try:
                    r = await client.get(f"{self.base_url}/health", timeout=5.0)
                    if r.status_code == 200:
                        break
                except httpx.HTTPError:
                    pass
                if time.monotonic() > deadline:
                    self.close()
                    raise TimeoutError(f"vLLM server not ready within {timeout_s:.0f} s (log: {self.log_path})")
                await asyncio.sleep(1.0)
            r = await client.get(f"{self.base_url}/v1/models", headers=self.headers(), timeout=10.0)
            r.raise_for_status()
        return self.base_url + "/v1"

    async def load_lora(self, name: str, path: str) -> None:
        """Serve the PEFT adapter at ``path`` as model ``name`` (hot load)."""
        import httpx

        async with httpx.AsyncClient() as client:
            if name in self.loaded:
                await self.unload_lora(name, client)
            r = await client.post(f"{self.base_url}/v1/load_lora_adapter", headers=self.headers(),
                                  json={"lora_name": name, "lora_path": os.path.abspath(path)}, timeout=120.0)
            if r.status_code >= 400:
                raise RuntimeError(f"vLLM refused adapter {name} at {path}: {r.status_code} {r.text[:300]}")
        self.loaded.add(name)

    async def unload_lora(self, name: str, client: Any = None) -> None:
        import httpx

        own = client is None
        client = client or httpx.AsyncClient()
        try:
            await client.post(f"{self.base_url}/v1/unload_lora_adapter", headers=self.headers(),
                              json={"lora_name": name}, timeout=60.0)
        finally:
            if own:
                await client.aclose()
        self.loaded.discard(name)

    def close(self) -> None:
        if self.process is not None:
            managed_process.stop_group(self.process, grace_s=20.0, kill_after_s=10.0)
            self.process = None
        if self._log is not None:
            self._log.close()
            self._log = None
        self.loaded.clear()

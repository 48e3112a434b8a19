"""OpenAI-compatible rollout server backed by the in-process generation engine.

The reference serves rollouts with vLLM behind an OpenAI-compatible API,
patched to return the prompt and completion token ids
(``src/art/vllm_runtime.py:218``, ``vllm_runtime/src/art_vllm_runtime/
dedicated_server.py:37-188``, ``patches.py``) and to hot-load each new LoRA
checkpoint under the name ``{model}@{step}``.  This server keeps that wire
contract on top of :class:`GenerationEngine`:

* ``GET /v1/models``; ``POST /v1/chat/completions`` and
  ``POST /v1/completions`` (``n``, ``max_tokens`` / ``max_completion_tokens``,
  ``temperature``, ``top_p``, ``seed``, ``stop``, ``logprobs``);
* every response carries ``prompt_token_ids`` (top level) and ``token_ids``
  (per choice) plus per-token logprobs, which is what the trainer's
  tokenizer consumes;
* model names: the live policy (the trainer's current adapter, shared in
  memory, so a finished training step is served immediately), ``{name}@{step}``
  of a saved checkpoint (loaded on first use), or the base model name;
* requests are batched: a worker thread drains the queue every few
  milliseconds and runs requests with the same adapter and sampling settings
  as one generation batch; ``engine_lock`` keeps generation and training
  steps of a colocated trainer from overlapping.
"""

from __future__ import annotations

import asyncio
import threading
import time
import uuid
from concurrent.futures import Future
from dataclasses import dataclass
from typing import Any, Callable

from fastapi import FastAPI, HTTPException, Request

from ..runtime.generate import GenerationEngine, SamplingParams


@dataclass
class _Job:
    prompt: list[int]
    params: SamplingParams
    adapter: str | None
    future: Future


class RolloutServer:
    def __init__(
        self,
        engine: GenerationEngine,
        tokenizer: Any,
        *,
        served_name: str,
        resolve_adapter: Callable[[str], str | None] | None = None,
        host: str = "127.0.0.1",
        port: int = 8000,
        api_key: str | None = None,
        batch_window_s: float = 0.005,
        max_batch: int = 256,
    ) -> None:
        self.engine, self.tokenizer = engine, tokenizer
        self.served_name = served_name
        self.resolve_adapter = resolve_adapter or (lambda name: None)
        self.host, self.port, self.api_key = host, port, api_key
        self.batch_window_s, self.max_batch = batch_window_s, max_batch
        self.engine_lock = threading.Lock()
        self._jobs: list[_Job] = []
        self._cv = threading.Condition()
        self._stop = False
        self._worker: threading.Thread | None = None
        self._server = None
        self._thread: threading.Thread | None = None

    # ------------------------------------------------------------------ batching
    def submit(self, prompt: list[int], params: SamplingParams, adapter: str | None) -> Future:
        f: Future = Future()
        with self._cv:
            self._jobs.append(_Job(prompt, params, adapter, f))
            self._cv.notify()
        return f

    def _work(self) -> None:
        while True:
            with self._cv:
                while not self._jobs and not self._stop:
                    self._cv.wait(0.1)
                if self._stop and not self._jobs:
                    return
            time.sleep(self.batch_window_s)  # let concurrent requests join the batch
            with self._cv:
                jobs, self._jobs = self._jobs[: self.max_batch], self._jobs[self.max_batch :]
            groups: dict[tuple, list[_Job]] = {}
            for j in jobs:
                p = j.params
                key = (j.adapter, p.max_tokens, p.temperature, p.top_p, tuple(p.stop_token_ids), p.seed)
                groups.setdefault(key, []).append(j)
            for batch in groups.values():
                try:
                    with self.engine_lock:
                        res = self.engine.generate([j.prompt for j in batch], batch[0].params, batch[0].adapter)
                    for j, r in zip(batch, res):
                        j.future.set_result(r)
                except Exception as exc:  # reported to every request of the batch
                    for j in batch:
                        if not j.future.done():
                            j.future.set_exception(exc)

    # ------------------------------------------------------------------ API
    def _params(self, body: dict[str, Any]) -> SamplingParams:
        stop_ids = list(getattr(self.tokenizer, "eos_token_ids", []))
        stop = body.get("stop_token_ids")
        if stop:
            stop_ids += [int(x) for x in stop]
        return SamplingParams(
            max_tokens=int(body.get("max_completion_tokens") or body.get("max_tokens") or 256),
            temperature=float(body.get("temperature", 1.0) if body.get("temperature") is not None else 1.0),
            top_p=float(body.get("top_p") or 1.0),
            stop_token_ids=stop_ids,
            seed=body.get("seed"),
        )

    async def _run(self, prompt: list[int], body: dict[str, Any]):
        name = body.get("model") or self.served_name
        adapter = self.resolve_adapter(name)
        params = self._params(body)
        n = int(body.get("n") or 1)
        futs = [self.submit(prompt, params, adapter) for _ in range(n)]
        return [await asyncio.wrap_future(f) for f in futs]

    def _logprobs(self, r) -> dict[str, Any]:
        tok = getattr(self.tokenizer, "token_str", lambda i: str(i))
        return {"content": [{"token": f"token_id:{t}", "logprob": lp, "bytes": list(tok(t).encode("utf-8", "replace")),
                             "top_logprobs": []} for t, lp in zip(r.token_ids, r.logprobs)]}

    async def chat_completions(self, body: dict[str, Any]) -> dict[str, Any]:
        prompt = self.tokenizer.apply_chat_template(body.get("messages") or [], tools=body.get("tools"))
        outs = await self._run(prompt, body)
        choices = []
        for i, r in enumerate(outs):
            text = self.tokenizer.decode([t for t in r.token_ids if t not in getattr(self.tokenizer, "eos_token_ids", [])])
            choices.append({
                "index": i, "finish_reason": r.finish_reason,
                "message": {"role": "assistant", "content": text},
                "logprobs": self._logprobs(r), "token_ids": r.token_ids,
            })
        comp = sum(len(r.token_ids) for r in outs)
        return {
            "id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion", "created": int(time.time()),
            "model": body.get("model") or self.served_name, "choices": choices, "prompt_token_ids": prompt,
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": comp, "total_tokens": len(prompt) + comp},
        }

    @staticmethod
    async def sse_chunks(out: dict[str, Any]):
        """A finished completion as server-sent chat.completion.chunk events:
        one content delta per choice (with its token ids and logprobs), then
        the finish reasons (generation here is not incremental)."""
        import json

        base = {"id": out["id"], "object": "chat.completion.chunk", "created": out["created"], "model": out["model"]}
        for ch in out["choices"]:
            delta = {"index": ch["index"], "delta": {"role": "assistant", "content": ch["message"]["content"]},
                     "logprobs": ch["logprobs"], "finish_reason": None, "token_ids": ch["token_ids"]}
            yield f"data: {json.dumps({**base, 'choices': [delta], 'prompt_token_ids': out['prompt_token_ids']})}\n\n"
        fin = [{"index": ch["index"], "delta": {}, "finish_reason": ch["finish_reason"]} for ch in out["choices"]]
        yield f"data: {json.dumps({**base, 'choices': fin, 'usage': out['usage']})}\n\n"
        yield "data: [DONE]\n\n"

    async def completions(self, body: dict[str, Any]) -> dict[str, Any]:
        p = body.get("prompt") or ""
        prompt = list(p) if isinstance(p, list) else self.tokenizer.encode(p)
        outs = await self._run(prompt, body)
        choices = [{
            "index": i, "text": self.tokenizer.decode(r.token_ids), "finish_reason": r.finish_reason,
            "logprobs": {"token_logprobs": r.logprobs, "tokens": [f"token_id:{t}" for t in r.token_ids]},
            "token_ids": r.token_ids,
        } for i, r in enumerate(outs)]
        comp = sum(len(r.token_ids) for r in outs)
        return {
            "id": f"cmpl-{uuid.uuid4().hex}", "object": "text_completion", "created": int(time.time()),
            "model": body.get("model") or self.served_name, "choices": choices, "prompt_token_ids": prompt,
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": comp, "total_tokens": len(prompt) + comp},
        }

    def app(self) -> FastAPI:
        app = FastAPI()
        server = self

        def check(req: Request) -> None:
            if server.api_key and req.headers.get("authorization") != f"Bearer {server.api_key}":
                raise HTTPException(status_code=401, detail="bad api key")

        @app.get("/v1/models")
        async def models(req: Request):
            check(req)
            names = [server.served_name, *server.engine.adapters]
            return {"object": "list", "data": [{"id": n, "object": "model", "owned_by": "art"} for n in names]}

        @app.post("/v1/chat/completions")
        async def chat(req: Request):
            check(req)
            body = await req.json()
            out = await server.chat_completions(body)
            if not body.get("stream"):
                return out
            from fastapi.responses import StreamingResponse

            return StreamingResponse(server.sse_chunks(out), media_type="text/event-stream")

        @app.post("/v1/completions")
        async def completions(req: Request):
            check(req)
            return await server.completions(await req.json())

        @app.get("/health")
        async def health():
            return {"ok": True}

        return app

    # ------------------------------------------------------------------ lifecycle
    def start(self, timeout_s: float = 30.0) -> None:
        import uvicorn

        self._worker = threading.Thread(target=self._work, name="rollout-engine", daemon=True)
        self._worker.start()
        cfg = uvicorn.Config(self.app(), host=self.host, port=self.port, log_level="warning")
        self._server = uvicorn.Server(cfg)
        self._thread = threading.Thread(target=self._server.run, name="rollout-http", daemon=True)
        self._thread.start()
        deadline = time.monotonic() + timeout_s
        while not self._server.started:
            if not self._thread.is_alive() or time.monotonic() > deadline:
                raise RuntimeError(f"rollout server did not start on {self.host}:{self.port}")
            time.sleep(0.01)

    def stop(self) -> None:
        if self._server is not None:
            self._server.should_exit = True
        if self._thread is not None:
            self._thread.join(10)
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        if self._worker is not None:
            self._worker.join(10)

    @property
    def base_url(self) -> str:
        return f"http://{self.host}:{self.port}/v1"

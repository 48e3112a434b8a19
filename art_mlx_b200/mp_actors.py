"""Run an object in a child process behind a proxy with the same interface.

Behaviour of the reference ``src/mp_actors/move.py:56-413``
(``move_to_child_process``, ``close_proxy``): method calls on the proxy are
forwarded to a pickled copy of the object living in a child process;
coroutine methods return awaitables, async-generator methods return async
generators (``asend`` supported), plain methods block and return their
result, other attributes are read from the child.  Exceptions raised in the
child are re-raised in the caller; if the child dies, every pending and
later call fails with an error naming its exit code or signal; the child
exits by itself when its parent process goes away.

Design for this framework: the child is started with the ``spawn`` method
(a CUDA context must never be forked), runs one asyncio loop that serves
requests concurrently (each request is a task, so a long async call does not
block the others) and talks over two ``multiprocessing`` queues; the parent
resolves ``concurrent.futures.Future`` objects from a dispatcher thread, so
the proxy works from any thread and any event loop.
"""

from __future__ import annotations

import asyncio
import inspect
import itertools
import multiprocessing as mp
import os
import queue
import sys
import threading
import time
import traceback
from concurrent.futures import Future
from dataclasses import dataclass, field
from typing import Any, TypeVar, cast

T = TypeVar("T")

_SHUTDOWN = -1


@dataclass
class _Request:
    id: int
    kind: str  # "call" | "getattr" | "agen_start" | "agen_next" | "agen_close"
    name: str = ""
    args: tuple = ()
    kwargs: dict = field(default_factory=dict)
    value: Any = None  # value sent into an async generator
    agen: int = 0  # async generator handle


@dataclass
class _Response:
    id: int
    result: Any = None
    error: BaseException | None = None
    tb: str = ""
    stop: bool = False  # async generator exhausted


class RemoteError(RuntimeError):
    """Wraps an exception raised in the child whose type cannot be re-raised."""


def _portable(exc: BaseException) -> BaseException:
    import pickle

    try:
        pickle.loads(pickle.dumps(exc))
        return exc
    except Exception:
        return RemoteError(f"{type(exc).__name__}: {exc}")


def _child(obj: Any, requests: Any, responses: Any, ready: Any, parent_pid: int, log_file: str | None,
           name: str | None) -> None:
    if log_file:
        f = open(log_file, "a", buffering=1)
        os.dup2(f.fileno(), sys.stdout.fileno())
        os.dup2(f.fileno(), sys.stderr.fileno())
    try:
        os.setpgid(0, 0)  # own process group: signals to the parent's group do not hit the child
    except OSError:
        pass

    def watch_parent() -> None:
        while True:
            if os.getppid() != parent_pid:
                os._exit(0)
            time.sleep(1.0)

    threading.Thread(target=watch_parent, daemon=True).start()
    ready.put(("ok", os.getpgid(0)))
    gens: dict[int, Any] = {}

    async def serve(req: _Request) -> None:
        resp = _Response(req.id)
        try:
            if req.kind == "getattr":
                resp.result = getattr(obj, req.name)
            elif req.kind == "call":
                out = getattr(obj, req.name)(*req.args, **req.kwargs)
                if inspect.isawaitable(out):
                    out = await out
                resp.result = out
            elif req.kind == "agen_start":
                gens[req.agen] = getattr(obj, req.name)(*req.args, **req.kwargs)
            elif req.kind == "agen_next":
                try:
                    resp.result = await gens[req.agen].asend(req.value)
                except StopAsyncIteration:
                    resp.stop = True
                    gens.pop(req.agen, None)
            elif req.kind == "agen_close":
                g = gens.pop(req.agen, None)
                if g is not None:
                    await g.aclose()
        except BaseException as exc:  # noqa: BLE001 - forwarded to the caller
            resp.error = _portable(exc)
            resp.tb = traceback.format_exc()
        responses.put(resp)

    async def loop() -> None:
        aio = asyncio.get_running_loop()
        tasks: set[asyncio.Task] = set()
        while True:
            req = await aio.run_in_executor(None, requests.get)
            if req.id == _SHUTDOWN:
                break
            t = asyncio.ensure_future(serve(req))
            tasks.add(t)
            t.add_done_callback(tasks.discard)
        for t in list(tasks):
            t.cancel()
        responses.put(_Response(_SHUTDOWN))

    asyncio.run(loop())


class Proxy:
    def __init__(self, obj: Any, log_file: str | None = None, process_name: str | None = None,
                 start_timeout: float | None = None) -> None:
        ctx = mp.get_context("spawn")
        self._obj_type = type(obj)
        self._probe = obj  # the parent's copy is used only to inspect method kinds
        self._name = process_name
        self._requests = ctx.Queue()
        self._responses = ctx.Queue()
        ready = ctx.Queue()
        self._process = ctx.Process(
            target=_child, args=(obj, self._requests, self._responses, ready, os.getpid(), log_file, process_name),
            name=process_name or "mp-actor", daemon=True,
        )
        self._process.start()
        limit = start_timeout if start_timeout is not None else float(os.environ.get("ART_MP_ACTOR_START_TIMEOUT", 300))
        deadline = time.monotonic() + limit
        while True:
            try:
                status, payload = ready.get(timeout=0.1)
                break
            except queue.Empty:
                if not self._process.is_alive():
                    raise self._death()
                if time.monotonic() > deadline:
                    self._process.kill()
                    raise RuntimeError(f"child process did not start within {limit:.0f}s")
        if status != "ok":
            raise RuntimeError(f"child process failed to start: {payload}")
        self._pgid = int(payload)
        self._futures: dict[int, Future] = {}
        self._lock = threading.Lock()
        self._ids = itertools.count(1)
        self._dead: RuntimeError | None = None
        self._closing = False
        self._dispatcher = threading.Thread(target=self._dispatch, name="mp-actor-dispatch", daemon=True)
        self._dispatcher.start()

    # ------------------------------------------------------------------
    def _death(self) -> RuntimeError:
        code = self._process.exitcode
        who = f" '{self._name}'" if self._name else ""
        if code is None:
            return RuntimeError(f"child process{who} died")
        if code < 0:
            return RuntimeError(f"child process{who} was killed by signal {-code}")
        return RuntimeError(f"child process{who} exited with code {code}")

    def _dispatch(self) -> None:
        while True:
            try:
                resp: _Response = self._responses.get(timeout=0.1)
            except queue.Empty:
                if self._closing:
                    return
                if self._dead is None and not self._process.is_alive():
                    self._dead = self._death()
                    with self._lock:
                        pending, self._futures = list(self._futures.values()), {}
                    for f in pending:
                        if not f.done():
                            f.set_exception(self._dead)
                continue
            except (EOFError, OSError):
                return
            if resp.id == _SHUTDOWN:
                return
            with self._lock:
                f = self._futures.pop(resp.id, None)
            if f is None or f.done():
                continue
            if resp.error is not None:
                f.set_exception(resp.error)
            else:
                f.set_result(resp)

    def _send(self, req: _Request) -> Future:
        f: Future = Future()
        with self._lock:
            if self._dead is not None:
                raise self._dead
            if self._closing:
                raise RuntimeError("proxy is closed")
            self._futures[req.id] = f
        self._requests.put(req)
        return f

    def _req(self, kind: str, **kw: Any) -> _Request:
        return _Request(id=next(self._ids), kind=kind, **kw)

    # ------------------------------------------------------------------
    def __getattr__(self, name: str) -> Any:
        if name.startswith("_"):
            raise AttributeError(name)
        attr = getattr(self._probe, name, None)
        if attr is None and not hasattr(self._probe, name):
            raise AttributeError(f"{self._obj_type.__name__} has no attribute {name!r}")
        if inspect.isasyncgenfunction(attr):
            return self._agen_method(name)
        if inspect.iscoroutinefunction(attr):
            async def acall(*args: Any, **kwargs: Any) -> Any:
                f = self._send(self._req("call", name=name, args=args, kwargs=kwargs))
                return (await asyncio.wrap_future(f)).result

            return acall
        if callable(attr):
            def call(*args: Any, **kwargs: Any) -> Any:
                return self._send(self._req("call", name=name, args=args, kwargs=kwargs)).result().result

            return call
        return self._send(self._req("getattr", name=name)).result().result

    def _agen_method(self, name: str):
        proxy = self

        def start(*args: Any, **kwargs: Any):
            handle = next(proxy._ids)
            proxy._send(proxy._req("agen_start", name=name, args=args, kwargs=kwargs, agen=handle)).result()

            class _Gen:
                def __aiter__(self):
                    return self

                async def __anext__(self):
                    return await self.asend(None)

                async def asend(self, value: Any):
                    f = proxy._send(proxy._req("agen_next", agen=handle, value=value))
                    resp = await asyncio.wrap_future(f)
                    if resp.stop:
                        raise StopAsyncIteration
                    return resp.result

                async def aclose(self):
                    await asyncio.wrap_future(proxy._send(proxy._req("agen_close", agen=handle)))

            return _Gen()

        return start

    def close(self, timeout: float = 10.0) -> None:
        if self._closing:
            return
        if self._process.is_alive():
            self._requests.put(_Request(id=_SHUTDOWN, kind="shutdown"))
            self._process.join(timeout)
        self._closing = True
        if self._process.is_alive():
            self._process.terminate()
            self._process.join(5)
        if self._process.is_alive():
            self._process.kill()
            self._process.join(5)
        with self._lock:
            pending, self._futures = list(self._futures.values()), {}
        for f in pending:
            if not f.done():
                f.set_exception(RuntimeError("proxy closed"))


def move_to_child_process(obj: T, log_file: str | None = None, process_name: str | None = None) -> T:
    """Move ``obj`` into a child process; returns a proxy with its interface."""
    return cast(T, Proxy(obj, log_file, process_name))


def close_proxy(proxy: object) -> None:
    """Stop the child process behind ``proxy`` (no-op for other objects)."""
    if isinstance(proxy, Proxy):
        proxy.close()

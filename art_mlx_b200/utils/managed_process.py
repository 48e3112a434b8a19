"""Child-process lifecycle: parent-death signal, process-group stop, watchdog.

Role of the reference's managed-process wrapper and lifecycle supervisor
(``src/art/utils/managed_process.py:24-101``, ``src/art/utils/lifecycle.py:68,148``):
a long-lived child (the multi-GPU worker group, a rollout server) must not
outlive the process that started it, must be stoppable together with
everything it spawned, and must not leave an awaiting caller blocked when it
dies on its own.

* :func:`popen` starts the child in its own session (so its whole process
  tree is one process group) and, on Linux, asks the kernel to send it
  ``SIGTERM`` when the parent's main thread exits (``prctl(PR_SET_PDEATHSIG)``).
  If the parent is already gone by the time the child runs, the child exits
  at once.
* :func:`stop_group` sends ``SIGTERM`` to the group, waits, then ``SIGKILL``.
  It only signals the group of a process this module started.
* :class:`Watchdog` polls a set of children from the event loop.  An exit that
  was not announced with :meth:`Watchdog.expect_exit` fails every coroutine
  running under :meth:`Watchdog.guard` with :class:`ChildProcessDied`.
"""

from __future__ import annotations

import asyncio
import ctypes
import os
import signal
import subprocess
import sys
import threading
from typing import Any, Awaitable, TypeVar

T = TypeVar("T")

_PR_SET_PDEATHSIG = 1


def _pdeathsig_preexec(sig: int, parent_pid: int):
    # resolved in the parent: between fork and exec the child must not enter the
    # dynamic loader (another thread of the parent may have held its lock at fork)
    try:
        prctl = ctypes.CDLL(None, use_errno=True).prctl
    except (OSError, AttributeError):
        return None

    def _fn() -> None:
        prctl(_PR_SET_PDEATHSIG, int(sig), 0, 0, 0)
        # the parent may have exited between fork and prctl: then nobody sends the signal
        if os.getppid() != parent_pid:
            os._exit(1)

    return _fn


def popen(cmd: list[str], *, die_with_parent: bool = True,
          death_signal: int = signal.SIGTERM, **kwargs: Any) -> subprocess.Popen:
    """``subprocess.Popen`` in a new session; with ``die_with_parent`` (Linux)
    the child gets ``death_signal`` when this process's main thread exits.
    The kernel ties the signal to the thread that forks, so it is only
    requested when called from the main thread (a child started from a
    short-lived thread would otherwise die with that thread)."""
    kwargs.setdefault("start_new_session", True)
    on_main = threading.current_thread() is threading.main_thread()
    if die_with_parent and on_main and sys.platform.startswith("linux"):
        if "preexec_fn" in kwargs:
            raise ValueError("popen sets preexec_fn itself")
        fn = _pdeathsig_preexec(death_signal, os.getpid())
        if fn is not None:
            kwargs["preexec_fn"] = fn
    return subprocess.Popen(cmd, **kwargs)


def stop_group(proc: subprocess.Popen, grace_s: float = 30.0, kill_after_s: float = 30.0) -> int | None:
    """Stop ``proc``'s process group (``proc`` must lead its own session, as
    :func:`popen` arranges): ``SIGTERM``, wait ``grace_s``, then ``SIGKILL``.
    Returns the exit code (None if the process could not be reaped)."""
    if proc.poll() is not None:
        return proc.returncode
    try:
        pgid = os.getpgid(proc.pid)
    except ProcessLookupError:
        return proc.poll()
    if pgid != proc.pid:
        raise ValueError("process does not lead its own process group; start it with managed_process.popen")
    for sig, wait_s in ((signal.SIGTERM, grace_s), (signal.SIGKILL, kill_after_s)):
        try:
            os.killpg(pgid, sig)
        except ProcessLookupError:
            break
        try:
            return proc.wait(timeout=wait_s)
        except subprocess.TimeoutExpired:
            continue
    return proc.poll()


class ChildProcessDied(RuntimeError):
    def __init__(self, name: str, returncode: int) -> None:
        how = f"was killed by signal {-returncode}" if returncode < 0 else f"exited with code {returncode}"
        super().__init__(f"child process {name!r} {how}")
        self.name, self.returncode = name, returncode


class Watchdog:
    """Polls registered children every ``interval_s`` seconds while at least
    one coroutine runs under :meth:`guard`."""

    def __init__(self, interval_s: float = 0.2) -> None:
        self.interval_s = interval_s
        self._procs: dict[str, subprocess.Popen] = {}
        self._expected: set[str] = set()
        self.failure: ChildProcessDied | None = None

    def add(self, name: str, proc: subprocess.Popen) -> None:
        self._procs[name] = proc
        self._expected.discard(name)

    def remove(self, name: str) -> None:
        self._procs.pop(name, None)
        self._expected.discard(name)

    def expect_exit(self, name: str) -> None:
        """Announce an intended stop: the exit of ``name`` is no failure."""
        self._expected.add(name)

    def check(self) -> None:
        """Raise :class:`ChildProcessDied` for the first child that exited
        unannounced (also usable without an event loop)."""
        if self.failure is not None:
            raise self.failure
        for name, proc in self._procs.items():
            code = proc.poll()
            if code is not None and name not in self._expected:
                self.failure = ChildProcessDied(name, code)
                raise self.failure

    async def _watch(self) -> None:
        while True:
            self.check()
            await asyncio.sleep(self.interval_s)

    async def guard(self, aw: Awaitable[T]) -> T:
        """Await ``aw``; if a watched child dies first, cancel it and raise."""
        self.check()
        work = asyncio.ensure_future(aw)
        watch = asyncio.ensure_future(self._watch())
        try:
            done, _ = await asyncio.wait({work, watch}, return_when=asyncio.FIRST_COMPLETED)
            if work in done:
                return work.result()
            work.cancel()
            try:
                await work
            except (asyncio.CancelledError, Exception):
                pass
            watch.result()  # raises ChildProcessDied
            raise AssertionError("watchdog ended without a failure")
        finally:
            watch.cancel()
            if not work.done():
                work.cancel()

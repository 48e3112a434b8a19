"""Child-process lifecycle (host only): parent-death signal, process-group
stop, and the asyncio watchdog (role of ``src/art/utils/managed_process.py``
and ``src/art/utils/lifecycle.py`` in the reference)."""

from __future__ import annotations

import asyncio
import os
import subprocess
import sys
import textwrap
import time

import pytest

from art_mlx_b200.utils import managed_process as mp

pytestmark = pytest.mark.skipif(not sys.platform.startswith("linux"), reason="prctl / process groups")


def _gone(pid: int) -> bool:
    """True once ``pid`` has exited (a zombie that nobody reaped counts as gone)."""
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().rsplit(")", 1)[1].split()[0] in ("Z", "X")
    except FileNotFoundError:
        return True


def _wait_gone(pid: int, limit_s: float = 10.0) -> bool:
    end = time.monotonic() + limit_s
    while time.monotonic() < end:
        if _gone(pid):
            return True
        time.sleep(0.05)
    return False


def test_child_dies_with_its_parent():
    # an intermediate process starts a managed child, reports its pid and exits
    script = textwrap.dedent(f"""
        import sys, time
        sys.path.insert(0, {os.getcwd()!r})
        from art_mlx_b200.utils import managed_process as mp
        p = mp.popen([sys.executable, "-c", "import time; time.sleep(60)"])
        print(p.pid, flush=True)
        time.sleep(0.5)
    """)
    out = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    child = int(out.stdout.split()[0])
    assert _wait_gone(child), "managed child outlived its parent"


def test_child_without_death_signal_survives_its_parent():
    script = textwrap.dedent(f"""
        import subprocess, sys
        sys.path.insert(0, {os.getcwd()!r})
        from art_mlx_b200.utils import managed_process as mp
        p = mp.popen([sys.executable, "-c", "import time; time.sleep(60)"], die_with_parent=False,
                     stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        print(p.pid, flush=True)
    """)
    out = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=60)
    child = int(out.stdout.split()[0])
    try:
        time.sleep(0.5)
        assert not _gone(child)
    finally:
        os.killpg(child, 9)  # the group this test's script started
    assert _wait_gone(child)


def test_stop_group_ends_the_whole_tree():
    # the child starts a grandchild in the same process group and prints its pid
    code = ("import subprocess, sys, time\n"
            "g = subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(60)'])\n"
            "print(g.pid, flush=True)\n"
            "time.sleep(60)\n")
    p = mp.popen([sys.executable, "-c", code], stdout=subprocess.PIPE, text=True)
    grandchild = int(p.stdout.readline())
    rc = mp.stop_group(p, grace_s=10)
    assert rc is not None and rc != 0
    assert _wait_gone(grandchild)


def test_stop_group_refuses_a_foreign_group():
    p = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])  # our own group
    try:
        with pytest.raises(ValueError):
            mp.stop_group(p)
    finally:
        p.kill()
        p.wait()


def test_watchdog_fails_the_guarded_call_when_a_child_dies():
    async def main():
        wd = mp.Watchdog(interval_s=0.05)
        p = mp.popen([sys.executable, "-c", "import time, sys; time.sleep(0.3); sys.exit(3)"])
        wd.add("worker", p)
        t0 = time.monotonic()
        with pytest.raises(mp.ChildProcessDied) as ei:
            await wd.guard(asyncio.sleep(30))
        assert ei.value.returncode == 3 and ei.value.name == "worker"
        assert time.monotonic() - t0 < 10
        with pytest.raises(mp.ChildProcessDied):  # sticky
            wd.check()

    asyncio.run(main())


def test_watchdog_ignores_an_announced_exit_and_returns_results():
    async def main():
        wd = mp.Watchdog(interval_s=0.05)
        p = mp.popen([sys.executable, "-c", "import time; time.sleep(60)"])
        wd.add("server", p)

        async def work():
            await asyncio.sleep(0.1)
            return 7

        assert await wd.guard(work()) == 7
        wd.expect_exit("server")
        mp.stop_group(p, grace_s=10)
        assert await wd.guard(work()) == 7

    asyncio.run(main())


def test_child_started_from_a_worker_thread_outlives_that_thread():
    import threading

    box = {}
    t = threading.Thread(target=lambda: box.setdefault(
        "p", mp.popen([sys.executable, "-c", "import time; time.sleep(60)"])))
    t.start()
    t.join()
    p = box["p"]
    try:
        time.sleep(0.5)
        assert p.poll() is None  # no death signal tied to the finished thread
    finally:
        mp.stop_group(p, grace_s=10)

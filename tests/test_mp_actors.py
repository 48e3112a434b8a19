"""The child-process proxy: sync, async and async-generator methods,
attribute reads, remote exceptions, concurrency and a dying child."""

import asyncio
import os

import pytest

from art_mlx_b200.mp_actors import close_proxy, move_to_child_process


class Counter:
    def __init__(self, start: int) -> None:
        self.value = start

    def add(self, n: int) -> int:
        self.value += n
        return self.value

    def pid(self) -> int:
        return os.getpid()

    async def slow_echo(self, x, delay: float):
        await asyncio.sleep(delay)
        return x

    async def count(self, n: int):
        got = 0
        for i in range(n):
            sent = yield i + got
            got = sent or 0

    def fail(self) -> None:
        raise ValueError("boom")

    def die(self) -> None:
        os._exit(7)


def test_proxy_methods_and_errors():
    p = move_to_child_process(Counter(10), process_name="counter")
    try:
        assert p.pid() != os.getpid()
        assert p.add(5) == 15 and p.add(1) == 16
        assert p.value == 16

        async def go():
            # concurrent async calls overlap in the child
            t0 = asyncio.get_running_loop().time()
            r = await asyncio.gather(*(p.slow_echo(i, 0.5) for i in range(4)))
            assert r == [0, 1, 2, 3]
            assert asyncio.get_running_loop().time() - t0 < 1.5
            out = []
            gen = p.count(3)
            out.append(await gen.__anext__())
            out.append(await gen.asend(10))
            out.append(await gen.asend(0))
            with pytest.raises(StopAsyncIteration):
                await gen.__anext__()
            assert out == [0, 11, 2]
            assert [x async for x in p.count(3)] == [0, 1, 2]

        asyncio.run(go())
        with pytest.raises(ValueError, match="boom"):
            p.fail()
    finally:
        close_proxy(p)


def test_dead_child_fails_pending_and_later_calls():
    p = move_to_child_process(Counter(0), process_name="doomed")
    try:
        with pytest.raises(RuntimeError, match="exited with code 7"):
            p.die()
        with pytest.raises(RuntimeError, match="exited with code 7"):
            p.add(1)
    finally:
        close_proxy(p)

"""Processor pool: results, per-task timeout with worker restart, crash recovery, error propagation."""

import asyncio
import os
import time

import pytest

from axrl_b200.processor.processor_pool import ProcessorCrashed, ProcessorPool, ProcessorTimeout


def _factory():
    def fn(x):
        if x == "sleep":
            time.sleep(30)
        if x == "crash":
            os._exit(3)
        if x == "raise":
            raise ValueError("bad input")
        return x * 2

    return fn


def test_pool_paths():
    async def go():
        pool = ProcessorPool(_factory, size=2, timeout_s=1.0)
        try:
            assert await asyncio.gather(*(pool.run(i) for i in range(6))) == [0, 2, 4, 6, 8, 10]
            with pytest.raises(ProcessorTimeout):
                await pool.run("sleep")
            with pytest.raises(ProcessorCrashed):
                await pool.run("crash")
            with pytest.raises(RuntimeError, match="bad input"):
                await pool.run("raise")
            assert await pool.run(21) == 42  # pool healthy after restarts
            assert pool.restarts == 2
        finally:
            pool.close()

    asyncio.run(go())

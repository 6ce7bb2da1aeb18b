"""Subprocess pool for CPU-side processors (tokenisers, verifiers, trace packing).

Reference: ``ProcessorPool`` (``axrl/processor/processor_pool.py:54-266``): work runs in child
processes so a hung or crashing verifier cannot take the rollout loop down; each task has a
timeout after which the worker is killed and restarted; a generation counter discards stale
results from a replaced worker; children die with their parent (``PR_SET_PDEATHSIG``).
"""

from __future__ import annotations

import asyncio
import ctypes
import itertools
import multiprocessing as mp
import os
import signal
from typing import Any, Callable


class ProcessorTimeout(Exception):
    pass


class ProcessorCrashed(Exception):
    pass


def _set_pdeathsig() -> None:
    try:
        libc = ctypes.CDLL("libc.so.6", use_errno=True)
        libc.prctl(1, signal.SIGKILL)  # PR_SET_PDEATHSIG
    except OSError:
        pass


def _worker_main(conn, factory: Callable[[], Callable[[Any], Any]]) -> None:  # noqa: ANN001
    _set_pdeathsig()
    fn = factory()
    while True:
        try:
            msg = conn.recv()
        except EOFError:
            return
        if msg is None:
            return
        tid, arg = msg
        try:
            conn.send((tid, True, fn(arg)))
        except Exception as e:  # noqa: BLE001
            conn.send((tid, False, f"{type(e).__name__}: {e}"))


class _Worker:
    def __init__(self, ctx, factory) -> None:  # noqa: ANN001
        self.parent, child = ctx.Pipe()
        self.proc = ctx.Process(target=_worker_main, args=(child, factory), daemon=True)
        self.proc.start()
        child.close()
        self.generation = 0

    def kill(self) -> None:
        if self.proc.is_alive():
            self.proc.kill()
        self.proc.join(timeout=5)
        self.parent.close()


class ProcessorPool:
    """``await pool.run(arg)`` executes ``factory()(arg)`` in one of ``size`` child processes."""

    def __init__(self, factory: Callable[[], Callable[[Any], Any]], size: int = 2, timeout_s: float = 30.0) -> None:
        self.ctx = mp.get_context("fork")
        self.factory, self.timeout_s = factory, timeout_s
        self.workers = [_Worker(self.ctx, factory) for _ in range(size)]
        self.idle: asyncio.Queue | None = None
        self.ids = itertools.count()
        self.restarts = 0

    async def _idle(self) -> asyncio.Queue:
        if self.idle is None:
            self.idle = asyncio.Queue()
            for i in range(len(self.workers)):
                self.idle.put_nowait(i)
        return self.idle

    def _restart(self, i: int) -> None:
        self.workers[i].kill()
        gen = self.workers[i].generation + 1
        self.workers[i] = _Worker(self.ctx, self.factory)
        self.workers[i].generation = gen
        self.restarts += 1

    async def run(self, arg: Any) -> Any:
        idle = await self._idle()
        i = await idle.get()
        w = self.workers[i]
        tid = next(self.ids)
        loop = asyncio.get_running_loop()
        try:
            w.parent.send((tid, arg))
            deadline = loop.time() + self.timeout_s
            while True:
                if await loop.run_in_executor(None, w.parent.poll, 0.05):
                    try:
                        rtid, ok, val = w.parent.recv()
                    except (EOFError, OSError):
                        self._restart(i)
                        raise ProcessorCrashed(f"processor worker {i} died") from None
                    if rtid != tid:  # stale answer from before a restart
                        continue
                    if not ok:
                        raise RuntimeError(val)
                    return val
                if not w.proc.is_alive():
                    self._restart(i)
                    raise ProcessorCrashed(f"processor worker {i} died")
                if loop.time() > deadline:
                    self._restart(i)
                    raise ProcessorTimeout(f"processor task exceeded {self.timeout_s}s")
        finally:
            idle.put_nowait(i)

    def close(self) -> None:
        for w in self.workers:
            try:
                w.parent.send(None)
            except (BrokenPipeError, OSError):
                pass
            w.kill()

    @staticmethod
    def pid_of(pool: "ProcessorPool", i: int) -> int:
        return pool.workers[i].proc.pid or os.getpid()

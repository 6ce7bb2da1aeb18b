"""Async task queues for the rollout control plane.

Reference counterpart: ``RemoteRayTaskQueue`` / ``RayTaskQueue`` (``axrl/utils/ray_task_queue.py:57-215``):
a queue with a global running limit, blocking ``get`` with timeout, ``complete`` to release a
running slot, and stats.  Here it is an asyncio object shared by coroutines of one process
(rollout loops, the controller); a process-level deployment puts it behind
:class:`axrl_b200.runtime.actors.ActorProxy`.
"""

from __future__ import annotations

import asyncio
import time
from collections import deque
from typing import Any, Generic, TypeVar

T = TypeVar("T")


class QueueClosed(Exception):
    pass


class AsyncTaskQueue(Generic[T]):
    def __init__(self, max_running: int | None = None, name: str = "queue") -> None:
        self.name = name
        self.max_running = max_running
        self._items: deque[T] = deque()
        self._cond = asyncio.Condition()
        self._running = 0
        self._closed = False
        self.stats = {"put": 0, "got": 0, "completed": 0, "timeouts": 0}
        self._created = time.time()

    async def put(self, item: T) -> None:
        await self.put_many([item])

    async def put_many(self, items: list[T]) -> None:
        async with self._cond:
            if self._closed:
                raise QueueClosed(self.name)
            self._items.extend(items)
            self.stats["put"] += len(items)
            self._cond.notify_all()

    def _can_take(self) -> bool:
        return bool(self._items) and (self.max_running is None or self._running < self.max_running)

    async def get(self, timeout: float | None = None) -> T | None:
        """Next item (counts as running until :meth:`complete`); None on timeout."""
        async with self._cond:
            try:
                await asyncio.wait_for(self._cond.wait_for(lambda: self._can_take() or self._closed), timeout)
            except asyncio.TimeoutError:
                self.stats["timeouts"] += 1
                return None
            if self._closed and not self._items:
                raise QueueClosed(self.name)
            self._running += 1
            self.stats["got"] += 1
            return self._items.popleft()

    async def complete(self, n: int = 1) -> None:
        async with self._cond:
            self._running = max(0, self._running - n)
            self.stats["completed"] += n
            self._cond.notify_all()

    async def close(self) -> None:
        async with self._cond:
            self._closed = True
            self._cond.notify_all()

    def qsize(self) -> int:
        return len(self._items)

    @property
    def running(self) -> int:
        return self._running

    def get_stats(self) -> dict[str, Any]:
        return {**self.stats, "pending": len(self._items), "running": self._running, "name": self.name}

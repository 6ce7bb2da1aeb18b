"""Rollout actors: N concurrent loops that pull conversations, run the recipe, and push results.

Reference: ``RemoteRolloutActor`` (``axrl/pipeline/rollout_actor.py:27-179``).  Each loop takes a
conversation from the rollout queue, runs ``recipe.run_rollout(conv, runtime)`` (which drives the
env/agent turn loop against the rollout worker), packs the finished trace into training samples
and pushes a :class:`RolloutResult` to the result queue.  Exceptions are kept and re-raised by
:meth:`check_health` so the controller can fail fast when a loop dies.
"""

from __future__ import annotations

import asyncio
import logging
from dataclasses import dataclass, field
from typing import Any

from axrl_b200.runtime.task_queue import AsyncTaskQueue, QueueClosed

logger = logging.getLogger(__name__)


@dataclass
class RolloutRuntime:
    """Handles a recipe's ``run_rollout`` may use (reference ``axrl/pipeline/rollout_data.py:22-64``)."""

    rollout_worker: Any
    local_processors: dict = field(default_factory=dict)
    shared_workers: dict = field(default_factory=dict)
    config: Any = None


@dataclass
class RolloutGroup:
    group_id: str
    results: list = field(default_factory=list)
    size: int = 0

    @property
    def complete(self) -> bool:
        return len(self.results) >= self.size


class RolloutActor:
    def __init__(self, recipe: Any, runtime: RolloutRuntime, rollout_queue: AsyncTaskQueue, result_queue: AsyncTaskQueue,
                 num_loops: int = 16, name: str = "rollout-actor") -> None:
        self.recipe, self.runtime = recipe, runtime
        self.rq, self.out = rollout_queue, result_queue
        self.num_loops = num_loops
        self.name = name
        self.tasks: list[asyncio.Task] = []
        self.error: BaseException | None = None
        self.completed = 0

    def start(self) -> None:
        self.tasks = [asyncio.create_task(self._loop(i)) for i in range(self.num_loops)]

    async def _loop(self, i: int) -> None:
        while True:
            try:
                conv = await self.rq.get(timeout=1.0)
            except QueueClosed:
                return
            if conv is None:
                continue
            try:
                result = await self.recipe.run_rollout(conv, self.runtime)
                await self.out.put(result)
                self.completed += 1
            except Exception as e:  # noqa: BLE001
                logger.exception("%s loop %d failed", self.name, i)
                self.error = e
                return
            finally:
                await self.rq.complete()

    def check_health(self) -> None:
        if self.error is not None:
            raise RuntimeError(f"{self.name} failed") from self.error
        dead = [t for t in self.tasks if t.done() and t.exception() is not None]
        if dead:
            raise RuntimeError(f"{self.name}: a rollout loop died") from dead[0].exception()

    async def stop(self) -> None:
        for t in self.tasks:
            t.cancel()
        await asyncio.gather(*self.tasks, return_exceptions=True)

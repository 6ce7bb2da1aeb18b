"""Least-loaded routing with session affinity across rollout engines.

Reference: ``InferenceRouter._assign_worker_index`` (``axrl/worker/infer_router.py:126-147``):
a session sticks to the engine that holds its KV prefix unless that engine is more than
``max_imbalance`` requests busier than the least-loaded one; new sessions go to the least
loaded engine.  Also warns when driver<->worker hand-off overhead exceeds a threshold
(reference :21,29-39).
"""

from __future__ import annotations

import logging
from typing import Any, Awaitable, Callable, Sequence

logger = logging.getLogger(__name__)

HANDOFF_WARN_SECONDS = 3.0


class InferenceRouter:
    def __init__(self, workers: Sequence[Any], max_imbalance: int = 16) -> None:
        assert workers, "need at least one engine"
        self.workers = list(workers)
        self.max_imbalance = max_imbalance
        self.load = [0] * len(workers)
        self.affinity: dict[str, int] = {}

    def assign(self, session_id: str | None) -> int:
        least = min(range(len(self.load)), key=lambda i: (self.load[i], i))
        if session_id is not None and session_id in self.affinity:
            i = self.affinity[session_id]
            if self.load[i] - self.load[least] <= self.max_imbalance:
                return i
        if session_id is not None:
            self.affinity[session_id] = least
        return least

    def release_session(self, session_id: str) -> None:
        self.affinity.pop(session_id, None)

    async def generate(self, inp: Any) -> Any:
        i = self.assign(getattr(inp, "session_id", None))
        self.load[i] += 1
        try:
            out = await self.workers[i].generate(inp)
        finally:
            self.load[i] -= 1
        ov = getattr(getattr(out, "event_timing", None), "overhead_seconds", lambda: None)()
        if ov is not None and ov > HANDOFF_WARN_SECONDS:
            logger.warning("driver<->engine hand-off overhead %.2fs for session %s", ov, getattr(inp, "session_id", "?"))
        return out

    async def broadcast(self, fn: Callable[[Any], Awaitable[Any]]) -> list[Any]:
        return [await fn(w) for w in self.workers]

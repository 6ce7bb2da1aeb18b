"""Rank liveness: heartbeats through the rendezvous store and bounded collectives.

Reference gap this fills: the reference fails the whole job when a rank dies, detecting it only
through the 1800 s NCCL timeout (``axrl/configs.py:385``).  Here every rank writes a heartbeat key
into the ``torch.distributed`` store from a daemon thread; :meth:`HeartbeatMonitor.check` (called
by the host between steps, before launching collectives) raises :class:`RankFailure` naming the
ranks whose heartbeat is older than ``timeout_s`` or that announced an exit.  Collective calls can
additionally be bounded with :func:`bounded_collective`, which runs the call asynchronously and
raises if it has not completed in time (the process group is then unusable and the job restarts
from its last checkpoint).
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable


class RankFailure(RuntimeError):
    def __init__(self, ranks: list[int], why: str) -> None:
        super().__init__(f"rank(s) {ranks} {why}")
        self.ranks = ranks


class HeartbeatMonitor:
    def __init__(self, store: Any, rank: int, world: int, interval_s: float = 1.0, timeout_s: float = 10.0, prefix: str = "axrl/hb") -> None:
        self.store, self.rank, self.world = store, rank, world
        self.interval_s, self.timeout_s, self.prefix = interval_s, timeout_s, prefix
        self._stop = threading.Event()
        self._th: threading.Thread | None = None
        self.t_start = time.time()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - the store went away: peers will notice our silence
                return
            self._stop.wait(self.interval_s)

    def start(self) -> "HeartbeatMonitor":
        self.beat()
        self._th = threading.Thread(target=self._loop, name="axrl-heartbeat", daemon=True)
        self._th.start()
        return self

    def stop(self, announce_exit: bool = True) -> None:
        self._stop.set()
        if self._th is not None:
            self._th.join(timeout=5)
        if announce_exit:
            try:
                self.store.set(self._key(self.rank), "exit")
            except Exception:  # noqa: BLE001
                pass

    def status(self) -> dict[int, float | str | None]:
        out: dict[int, float | str | None] = {}
        for r in range(self.world):
            try:
                v = self.store.get(self._key(r)).decode() if self.store.check([self._key(r)]) else None
            except Exception:  # noqa: BLE001
                v = None
            out[r] = v if v in (None, "exit") else float(v)
        return out

    def check(self) -> None:
        """Raise RankFailure if a peer exited or its heartbeat is stale."""
        now = time.time()
        exited, stale = [], []
        for r, v in self.status().items():
            if r == self.rank:
                continue
            if v == "exit":
                exited.append(r)
            elif v is None:
                if now - self.t_start > self.timeout_s:
                    stale.append(r)  # never joined
            elif now - v > self.timeout_s:
                stale.append(r)
        if exited:
            raise RankFailure(exited, "left the job")
        if stale:
            raise RankFailure(stale, f"sent no heartbeat for more than {self.timeout_s:.0f}s")


def bounded_collective(fn: Callable[..., Any], *args: Any, timeout_s: float = 60.0, **kw: Any) -> Any:
    """Run an async-capable ``torch.distributed`` collective and wait at most ``timeout_s``."""
    work = fn(*args, async_op=True, **kw)
    t0 = time.time()
    while not work.is_completed():
        if time.time() - t0 > timeout_s:
            raise TimeoutError(f"collective {getattr(fn, '__name__', fn)} did not complete within {timeout_s}s")
        time.sleep(0.005)
    work.wait()
    return work

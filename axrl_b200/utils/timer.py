"""Timers with JSON-tagged log lines, and GPU usage tracking.

Reference: ``Timer`` / ``SessionTimer`` (``axrl/utils/timer.py:10-101``) and ``GpuUsageTracker``
(``axrl/utils/gpu_utils.py:63-97``).  Device time is measured with CUDA events (never wall clock
for GPU work); ``GpuUsageTracker`` records wall time plus peak allocated/reserved memory.
"""

from __future__ import annotations

import json
import logging
import time
from dataclasses import dataclass

import torch

logger = logging.getLogger("axrl_b200.timer")


class Timer:
    def __init__(self, name: str = "", verbose: bool = True) -> None:
        self.name, self.verbose = name, verbose
        self.elapsed_seconds = 0.0

    def __enter__(self) -> "Timer":
        self.t0 = time.perf_counter()
        if self.verbose:
            logger.info("start %s", self.name)
        return self

    def __exit__(self, *exc) -> None:  # noqa: ANN002
        self.elapsed_seconds = time.perf_counter() - self.t0
        if self.verbose:
            logger.info("finish %s in %.3fs", self.name, self.elapsed_seconds)


class SessionTimer(Timer):
    """Timer whose log lines embed ``{session_id, execution_kind, function_name}`` as JSON (for timelines).

    When ``AXRL_SESSION_TIMELINE`` names a file, every finished span is also appended to it as one
    JSON line ``{session_id, execution_kind, function_name, start, end}`` (wall-clock seconds) —
    the input of :mod:`axrl_b200.utils.visualize_session_timer`."""

    def __init__(self, session_id: str, execution_kind: str, function_name: str) -> None:
        self.tag = {"session_id": session_id, "execution_kind": execution_kind, "function_name": function_name}
        super().__init__(json.dumps(self.tag))

    def __enter__(self) -> "SessionTimer":
        self.wall0 = time.time()
        super().__enter__()
        return self

    def __exit__(self, *exc) -> None:  # noqa: ANN002
        super().__exit__(*exc)
        import os

        path = os.environ.get("AXRL_SESSION_TIMELINE")
        if path:
            with open(path, "a") as f:
                f.write(json.dumps({**self.tag, "start": self.wall0, "end": self.wall0 + self.elapsed_seconds}) + "\n")


class CudaTimer:
    """Device time of the enclosed stream work (CUDA events on the current stream)."""

    def __enter__(self) -> "CudaTimer":
        self.s, self.e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.s.record()
        return self

    def __exit__(self, *exc) -> None:  # noqa: ANN002
        self.e.record()
        self.e.synchronize()
        self.ms = self.s.elapsed_time(self.e)


@dataclass
class GpuUsageInfo:
    name: str
    wall_s: float
    peak_mem_gbs: float
    peak_mem_reserved_gbs: float

    def to_metrics(self) -> dict[str, float]:
        return {"cpu_time_s": self.wall_s, "peak_mem_gbs": self.peak_mem_gbs, "peak_mem_reserved_gbs": self.peak_mem_reserved_gbs}


class GpuUsageTracker:
    def __init__(self, name: str) -> None:
        self.name = name
        self.usage_info: GpuUsageInfo | None = None

    def __enter__(self) -> "GpuUsageTracker":
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats()
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc) -> None:  # noqa: ANN002
        cuda = torch.cuda.is_available()
        if cuda:
            torch.cuda.synchronize()
        g = 1 << 30
        self.usage_info = GpuUsageInfo(self.name, time.perf_counter() - self.t0,
                                       torch.cuda.max_memory_allocated() / g if cuda else 0.0,
                                       torch.cuda.max_memory_reserved() / g if cuda else 0.0)

"""NVTX ranges for the pipeline phases (rollout, prefill, decode bursts, micro-batch
forward/backward, optimizer, weight sync) and CUDA memory-history snapshots.

The reference has no profiler integration; it exposes ``torch.cuda.memory._record_memory_history``
/ ``_dump_snapshot`` per rank (``axrl/worker/megatron_worker.py:376-384``).  Ranges are no-ops unless
``AXRL_NVTX=1`` (so production runs pay nothing); they nest and show up in Nsight timelines.
"""

from __future__ import annotations

import contextlib
import os
from typing import Iterator

import torch

_ON = os.environ.get("AXRL_NVTX", "0") == "1"


def enabled() -> bool:
    return _ON and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def start_memory_history(max_entries: int = 100_000) -> None:
    """Record allocator events (stack traces included) for a later snapshot."""
    if torch.cuda.is_available():
        torch.cuda.memory._record_memory_history(max_entries=max_entries)


def dump_memory_snapshot(path: str) -> None:
    """Write the recorded allocator history (open it with PyTorch's memory viz)."""
    if torch.cuda.is_available():
        torch.cuda.memory._dump_snapshot(path)
        torch.cuda.memory._record_memory_history(enabled=None)

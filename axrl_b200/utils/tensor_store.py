"""Handle-based tensor store (the host data plane).

Reference: ``TensorHandle`` / ``put`` / ``get_batch`` / ``delete_batch`` over Ray plasma
(``axrl/utils/tensor_store.py:27-91``).  Producers (rollout workers capturing routed experts)
``put`` an array and pass a small :class:`TensorHandle` through the control plane; consumers
(the trainer's routing materialiser) ``get_batch`` many handles at once — duplicate refs are read
once and row-sliced views are returned — and ``delete_batch`` frees them.

Two backends: in-process (a dict, for single-process deployments) and shared memory (one POSIX
segment per object through the native ``ShmSegment``, optionally page-locked so the trainer's
host-to-device copies are asynchronous).
"""

from __future__ import annotations

import itertools
import os
from dataclasses import dataclass
from typing import Sequence

import numpy as np


@dataclass(frozen=True)
class TensorHandle:
    ref: str
    row_start: int = 0
    row_count: int = -1  # -1: all rows from row_start

    def slice(self, start: int, count: int) -> "TensorHandle":
        base = self.row_start + start
        return TensorHandle(self.ref, base, count)


class TensorStore:
    def __init__(self, backend: str = "local", prefix: str | None = None, pin: bool = False) -> None:
        assert backend in ("local", "shm")
        self.backend, self.pin = backend, pin
        self.prefix = prefix or f"/axrl_{os.getpid()}"
        self._ids = itertools.count()
        self._local: dict[str, np.ndarray] = {}
        self._segs: dict[str, object] = {}
        self._meta: dict[str, tuple] = {}

    def put(self, arr: np.ndarray) -> TensorHandle:
        arr = np.ascontiguousarray(arr)
        ref = f"{self.prefix}_{next(self._ids)}"
        if self.backend == "local":
            self._local[ref] = arr
        else:
            from axrl_b200.rollout.kv import runtime_module

            seg = runtime_module().ShmSegment(ref, max(arr.nbytes, 1), True)
            np.frombuffer(seg.view(), dtype=np.uint8)[: arr.nbytes] = arr.view(np.uint8).reshape(-1)
            if self.pin:
                seg.pin()
            self._segs[ref] = seg
        self._meta[ref] = (arr.dtype.str, arr.shape)
        return TensorHandle(ref, 0, arr.shape[0] if arr.ndim else 1)

    def _array(self, ref: str) -> np.ndarray:
        if ref in self._local:
            return self._local[ref]
        dt, shape = self._meta[ref]
        seg = self._segs[ref]
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        return np.frombuffer(seg.view(), dtype=np.uint8)[:n].view(np.dtype(dt)).reshape(shape)

    def get_batch(self, handles: Sequence[TensorHandle]) -> list[np.ndarray]:
        cache: dict[str, np.ndarray] = {}
        out = []
        for h in handles:
            if h.ref not in cache:
                cache[h.ref] = self._array(h.ref)
            a = cache[h.ref]
            end = a.shape[0] if h.row_count < 0 else h.row_start + h.row_count
            out.append(a[h.row_start:end])
        return out

    def delete_batch(self, handles: Sequence[TensorHandle]) -> None:
        for ref in {h.ref for h in handles}:
            self._local.pop(ref, None)
            seg = self._segs.pop(ref, None)
            if seg is not None:
                seg.close()
                seg.unlink()
            self._meta.pop(ref, None)

    def __len__(self) -> int:
        return len(self._meta)

"""Byte counters for host<->device traffic issued by the framework (per GRPO step reporting)."""

from __future__ import annotations

import torch

_C = {"h2d": 0, "d2h": 0}


def add_h2d(*tensors: torch.Tensor) -> None:
    _C["h2d"] += sum(int(t.numel() * t.element_size()) for t in tensors if t is not None)


def add_d2h(*tensors: torch.Tensor) -> None:
    _C["d2h"] += sum(int(t.numel() * t.element_size()) for t in tensors if t is not None)


def snapshot() -> tuple[int, int]:
    return _C["h2d"], _C["d2h"]


def reset() -> None:
    _C["h2d"] = _C["d2h"] = 0

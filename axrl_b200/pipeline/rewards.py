"""Group reward normalisation and zero-std filtering.

Reference: ``PipelineController.normalize_group_rewards``
(``axrl/pipeline/controller.py:867-904``): advantage = clip((s - mean) / (std + 1e-6), -5, 5)
with the sample std (ddof = 1), 0 when the group std is below 1e-8.
"""

from __future__ import annotations

import numpy as np


def group_advantages(scores: list[float] | np.ndarray) -> tuple[np.ndarray, float, float]:
    s = np.asarray(scores, dtype=np.float64)
    assert s.size > 1, "at least two rollouts per group are needed for group statistics"
    mean = float(s.mean())
    std = float(s.std(ddof=1))
    if std < 1e-8:
        return np.zeros_like(s), mean, std
    return np.clip((s - mean) / (std + 1e-6), -5.0, 5.0), mean, std


def is_zero_std_group(scores: list[float] | np.ndarray) -> bool:
    s = np.asarray(scores, dtype=np.float64)
    return s.size > 1 and float(s.std(ddof=1)) < 1e-8

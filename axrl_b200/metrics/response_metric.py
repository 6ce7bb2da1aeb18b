"""Per-response metrics and their aggregation (reference ``axrl/metrics/response_metric.py:15-231``).

Aggregated keys live under ``Valid-Rollouts/*`` / ``All-Rollouts/*`` and include
``throughput_tokens_per_second`` (reference :179).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np


@dataclass
class ResponseMetric:
    score: float | None = None
    score_mean: float | None = None
    score_std: float | None = None
    response_length: int = 0
    prompt_length: int = 0
    finish_reason: str = "stop"
    num_turns: int = 1
    elapsed_seconds: float = 0.0
    repetition_ratio: float = 0.0
    extra: dict = field(default_factory=dict)

    @staticmethod
    def repetition(tokens: Sequence[int], n: int = 4) -> float:
        if len(tokens) < n + 1:
            return 0.0
        grams = [tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1)]
        return 1.0 - len(set(grams)) / len(grams)


def aggregate_response_metrics(metrics: Sequence[ResponseMetric], prefix: str = "All-Rollouts", wall_seconds: float | None = None) -> dict[str, float]:
    if not metrics:
        return {}
    lens = np.asarray([m.response_length for m in metrics], dtype=np.float64)
    scores = np.asarray([m.score for m in metrics if m.score is not None], dtype=np.float64)
    out = {
        f"{prefix}/num": float(len(metrics)),
        f"{prefix}/response_length_mean": float(lens.mean()),
        f"{prefix}/response_length_max": float(lens.max()),
        f"{prefix}/response_length_min": float(lens.min()),
        f"{prefix}/turns_mean": float(np.mean([m.num_turns for m in metrics])),
        f"{prefix}/repetition_mean": float(np.mean([m.repetition_ratio for m in metrics])),
    }
    if scores.size:
        out[f"{prefix}/score_mean"] = float(scores.mean())
        out[f"{prefix}/score_std"] = float(scores.std())
    for reason in sorted({m.finish_reason for m in metrics}):
        out[f"{prefix}/finish_{reason}_ratio"] = float(np.mean([m.finish_reason == reason for m in metrics]))
    if wall_seconds:
        out[f"{prefix}/throughput_tokens_per_second"] = float(lens.sum() / wall_seconds)
    return out

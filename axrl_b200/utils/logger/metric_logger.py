"""Metric loggers (console / TensorBoard / W&B) and a cross-rank buffer.

Reference: ``axrl/utils/logger/*.py`` (``MetricLogger`` backends selected by
``MetricLoggerConfig.logger_type``; ``LoggerBuffer`` gathers per-step metrics over ranks and
aggregates by name suffix ``_max`` / ``_min`` / ``_sum`` / mean or an explicit aggregation type,
``logger_buffer.py:19-127``).
"""

from __future__ import annotations

import json
import logging
import sys
import time
from collections import defaultdict
from typing import Any

import numpy as np

logger = logging.getLogger("axrl_b200")


class MetricLogger:
    def log(self, step: int, metrics: dict[str, float]) -> None:
        raise NotImplementedError

    def close(self) -> None:
        pass


class ConsoleLogger(MetricLogger):
    def __init__(self, stream=sys.stdout) -> None:  # noqa: ANN001
        self.stream = stream

    def log(self, step: int, metrics: dict[str, float]) -> None:
        self.stream.write(json.dumps({"step": step, "time": time.time(), **{k: v for k, v in metrics.items() if isinstance(v, (int, float))}}) + "\n")
        self.stream.flush()


class TensorBoardLogger(MetricLogger):
    def __init__(self, log_dir: str) -> None:
        from torch.utils.tensorboard import SummaryWriter

        self.w = SummaryWriter(log_dir)

    def log(self, step: int, metrics: dict[str, float]) -> None:
        for k, v in metrics.items():
            if isinstance(v, (int, float)):
                self.w.add_scalar(k, v, step)

    def close(self) -> None:
        self.w.close()


class WandbLogger(MetricLogger):
    def __init__(self, project: str, name: str, group: str | None = None, run_id: str | None = None) -> None:
        import wandb  # optional dependency

        self.run = wandb.init(project=project, name=name, group=group, id=run_id, resume="allow")

    def log(self, step: int, metrics: dict[str, float]) -> None:
        self.run.log(metrics, step=step)

    def close(self) -> None:
        self.run.finish()


def make_metric_logger(cfg) -> MetricLogger:  # noqa: ANN001
    if cfg.logger_type == "tensorboard":
        return TensorBoardLogger(str(cfg.get_log_dir() / cfg.name))
    if cfg.logger_type == "wandb":
        return WandbLogger(cfg.project_name, cfg.name, cfg.group_name, cfg.run_id)
    return ConsoleLogger()


class LoggerBuffer:
    """Buffer per-step metrics, gather across ranks, aggregate by suffix or registered type."""

    def __init__(self, group: Any = None) -> None:
        self.group = group
        self.buf: dict[int, list[dict[str, float]]] = defaultdict(list)
        self.agg_types: dict[str, list[str]] = {}

    def set_metric_agg_type(self, name: str, types: list[str]) -> None:
        self.agg_types[name] = types

    def update_metrics(self, step: int, tag: str, metrics: list[dict[str, float]], gather_group: str | None = None) -> None:
        for m in metrics:
            self.buf[step].append({f"{tag}/{k}" if tag else k: v for k, v in m.items() if isinstance(v, (int, float))})

    def aggregate(self, rows: list[dict[str, float]]) -> dict[str, float]:
        vals: dict[str, list[float]] = defaultdict(list)
        for r in rows:
            for k, v in r.items():
                vals[k].append(float(v))
        out = {}
        for k, v in vals.items():
            base = k.rsplit("/", 1)[-1]
            if base in self.agg_types:
                for t in self.agg_types[base]:
                    out[f"{k}_{t}"] = float(getattr(np, t)(v))
            elif k.endswith("_max"):
                out[k] = max(v)
            elif k.endswith("_min"):
                out[k] = min(v)
            elif k.endswith("_sum"):
                out[k] = sum(v)
            else:
                out[k] = float(np.mean(v))
        return out

    def aggregate_step_metrics(self, rows: list[dict[str, float]]) -> dict[str, float]:
        return self.aggregate(rows)

    def sync_and_flush(self) -> tuple[int | None, dict[str, float]]:
        import torch.distributed as dist

        if not self.buf:
            return None, {}
        step = max(self.buf)
        rows = [r for s in sorted(self.buf) for r in self.buf[s]]
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            gathered: list[Any] = [None] * dist.get_world_size(self.group)
            dist.all_gather_object(gathered, rows, group=self.group)
            rows = [r for g in gathered for r in g]
        self.buf.clear()
        return step, self.aggregate(rows)

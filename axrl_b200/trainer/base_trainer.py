"""Masked aggregations shared by every trainer (reference ``axrl/trainer/base_trainer.py:92-162``)."""

from __future__ import annotations

import torch

from axrl_b200.configs import ValueAggType

_EPS = 1e-10


def denominator_count(mask: torch.Tensor, mode: ValueAggType) -> torch.Tensor:
    if mode == "token-mean":
        return mask.sum(dtype=torch.int)
    if mode == "seq-mean-token-mean":
        return (mask.sum(-1) > 0).sum(dtype=torch.int)
    raise ValueError(f"no denominator for mode {mode!r}")


def aggregate_with_mask(value: torch.Tensor, mask: torch.Tensor, mode: ValueAggType) -> torch.Tensor:
    """Reduce a (B, T) tensor over the masked tokens according to ``mode``."""
    assert value.shape == mask.shape, f"{value.shape} vs {mask.shape}"
    if mode == "token-mean":
        return (value * mask).sum() / (denominator_count(mask, mode) + _EPS)
    if mode == "seq-mean-token-mean":
        cnt = mask.sum(-1)
        per_seq = (value * mask).sum(-1) / (cnt + _EPS)
        return (per_seq * (cnt > 0)).sum() / (denominator_count(mask, mode) + _EPS)
    if mode == "token-max":
        return value.masked_fill(mask == 0, float("-inf")).max()
    if mode == "token-min":
        return value.masked_fill(mask == 0, float("inf")).min()
    if mode == "token-std":
        n = denominator_count(mask, "token-mean") + _EPS
        mu = (value * mask).sum() / n
        return torch.sqrt(((value - mu) ** 2 * mask).sum() / n + _EPS)
    if mode in ("token-p05", "token-p95"):
        sel = value[mask.bool()]
        if sel.numel() == 0:
            return torch.zeros((), device=value.device)
        return torch.quantile(sel.float(), 0.05 if mode == "token-p05" else 0.95)
    if mode == "seq-mean-token-std":
        mf = mask.float()
        ln = mf.sum(-1).clamp(min=1.0)
        mu = (value * mf).sum(-1) / ln
        sd = torch.sqrt((((value - mu[:, None]) ** 2) * mf).sum(-1) / ln + _EPS)
        valid = mf.sum(-1) > 0
        return (sd * valid).sum() / valid.sum().clamp(min=1)
    raise ValueError(f"unknown aggregation mode {mode!r}")


class BaseTrainer:
    aggregate_with_mask = staticmethod(aggregate_with_mask)
    compute_denominator_count = staticmethod(denominator_count)

    def set_metric_agg_type(self, logger_buffer) -> None:  # noqa: ANN001
        logger_buffer.set_metric_agg_type("peak_mem_reserved_gbs", ["min", "max"])
        logger_buffer.set_metric_agg_type("peak_mem_gbs", ["min", "max"])
        logger_buffer.set_metric_agg_type("cpu_time_s", ["mean", "std"])

    def loss_func(self, outputs: dict, batch) -> tuple:  # noqa: ANN001
        raise NotImplementedError

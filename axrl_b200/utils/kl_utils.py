"""KL estimators between per-token logprobs (reference ``axrl/utils/kl_utils.py:15-105``).

``r = logprobs - base`` per token (fp32):
  k1 = r, k2 = r**2 / 2, k3 = exp(-r) - 1 + r   (Schulman's estimators).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch

KLType = Literal["k1", "k2", "k3"]


def kl_divergence(logprobs: torch.Tensor, logprobs_ref: torch.Tensor, kl_type: KLType = "k2") -> torch.Tensor:
    r = logprobs.float() - logprobs_ref.float()
    if kl_type == "k1":
        return r
    if kl_type == "k2":
        return 0.5 * r * r
    if kl_type == "k3":
        return torch.expm1(-r) + r
    raise ValueError(f"unknown kl_type {kl_type!r}")


@dataclass
class LogprobsDiffResult:
    k1: float
    k1_max: float
    k2: float
    k2_max: float
    k3: float
    k3_max: float
    cosine_similarity: float
    base_logprobs_mean: float
    test_logprobs_mean: float


def compare_logprobs(loss_masks: torch.Tensor, base_logprobs: torch.Tensor, test_logprobs: torch.Tensor) -> LogprobsDiffResult:
    """Per-sequence KL / cosine statistics over loss-masked tokens, averaged over sequences."""
    assert len(base_logprobs) == len(test_logprobs)
    rows = []
    for base, test, m in zip(base_logprobs, test_logprobs, loss_masks, strict=True):
        n = len(base)
        m = torch.as_tensor(m)[:n].bool()
        if not m.any():
            continue
        b = torch.as_tensor(base, dtype=torch.float32)[m]
        t = torch.as_tensor(test, dtype=torch.float32)[m]
        k1, k2, k3 = (kl_divergence(t, b, k) for k in ("k1", "k2", "k3"))
        rows.append(
            (k1.abs().mean(), k1.abs().max(), k2.mean(), k2.abs().max(), k3.mean(), k3.abs().max(), b.mean(), t.mean(),
             torch.nn.functional.cosine_similarity(b[None], t[None]).squeeze())
        )
    assert rows, "no loss-masked tokens to compare"
    cols = list(zip(*rows))
    mean = lambda i: float(torch.stack(cols[i]).mean())  # noqa: E731
    mx = lambda i: float(torch.stack(cols[i]).max())  # noqa: E731
    return LogprobsDiffResult(
        k1=mean(0), k1_max=mx(1), k2=mean(2), k2_max=mx(3), k3=mean(4), k3_max=mx(5),
        cosine_similarity=mean(8), base_logprobs_mean=mean(6), test_logprobs_mean=mean(7),
    )

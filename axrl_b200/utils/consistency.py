"""Cross-rank consistency checks: tensors that must be identical on every rank of a group.

Reference counterpart: the reference's dense invariant asserts (token conservation through packing,
routing row counts, duplicate-index checks) and its determinism modes (``deterministic_mode``,
``batch_invariant_mode``, ``axrl/configs.py:437-438``) stand in for race detection.  Here replicated
state (data-parallel parameters after an optimizer step, TP-replicated norms, the router of an EP
group) is compared across ranks by checksum: a silent divergence (a race in a collective kernel, a
missed reduction, a rank that skipped an update) surfaces as an error naming the tensors instead of
as drift.

Enabled in the trainer by ``AXRL_CONSISTENCY_CHECKS=1`` (one small all-gather per step).
"""

from __future__ import annotations

import os
from typing import Any, Iterable

import torch
import torch.distributed as dist


def enabled() -> bool:
    return os.environ.get("AXRL_CONSISTENCY_CHECKS", "0") == "1"


def checksums(tensors: Iterable[torch.Tensor]) -> torch.Tensor:
    """(n, 2) float64: sum and sum of |x| * (1 + position weight) of each tensor (order sensitive)."""
    rows = []
    for t in tensors:
        x = t.detach().reshape(-1).double()
        w = torch.linspace(1.0, 2.0, x.numel(), dtype=torch.float64, device=x.device) if x.numel() > 1 else torch.ones_like(x)
        rows.append(torch.stack([x.sum(), (x.abs() * w).sum()]))
    return torch.stack(rows) if rows else torch.zeros(0, 2, dtype=torch.float64)


def check_replicated(named: Iterable[tuple[str, torch.Tensor]], group: Any = None, rtol: float = 0.0) -> None:
    """Raise ``RuntimeError`` naming every tensor whose checksum differs between the ranks of
    ``group`` (bit-identical tensors are expected by default: ``rtol=0``)."""
    named = list(named)
    if not named or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    local = checksums(t for _, t in named)
    dev = named[0][1].device
    if dist.get_backend(group) == "nccl" and dev.type != "cuda":
        dev = torch.device("cuda", torch.cuda.current_device())
    local = local.to(dev)
    parts = [torch.empty_like(local) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, local, group=group)
    allc = torch.stack(parts).cpu()  # (world, n, 2)
    ref = allc[0]
    tol = rtol * ref.abs().clamp(min=1.0)
    bad = ((allc - ref).abs() > tol).any(dim=2).any(dim=0)
    if bool(bad.any()):
        names = [named[i][0] for i in range(len(named)) if bool(bad[i])]
        raise RuntimeError(f"replicated tensors differ across ranks: {names[:8]}{' ...' if len(names) > 8 else ''}")

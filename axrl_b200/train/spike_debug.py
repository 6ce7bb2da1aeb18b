"""Gradient-spike detection and debug snapshots.

Reference: ``MegatronWorker._detect_spike`` / ``_snapshot_spike_debug_info``
(``axrl/worker/megatron_worker.py:511-596``) and the replay tooling: a spike is a grad norm
above ``spike_ratio`` x the median of the last ``history_window`` norms (after ``warmup_steps``).
The snapshot directory ``spike_snapshots/iter_XXXXXXX`` holds the model + optimizer checkpoint,
the input batch, per-parameter grad norms and metadata; the most recent ``max_snapshots`` are
kept.  :func:`replay_snapshot` reloads a snapshot and recomputes the gradient norm so a spike can
be reproduced and bisected offline.
"""

from __future__ import annotations

import json
import shutil
import statistics
from collections import deque
from pathlib import Path
from typing import Any

import torch

from axrl_b200.configs import GradSpikeDebugConfig


class SpikeDetector:
    def __init__(self, cfg: GradSpikeDebugConfig) -> None:
        self.cfg = cfg
        self.history: deque[float] = deque(maxlen=cfg.history_window)
        self.steps = 0

    def observe(self, grad_norm: float) -> bool:
        """Record ``grad_norm``; True when it is a spike (never during warm-up)."""
        self.steps += 1
        spike = False
        if self.cfg.enabled and self.steps > self.cfg.warmup_steps and len(self.history) >= 2:
            spike = grad_norm > self.cfg.spike_ratio * statistics.median(self.history)
        if grad_norm == grad_norm and grad_norm != float("inf"):
            self.history.append(grad_norm)
        return spike


def per_param_grad_norms(model: torch.nn.Module) -> dict[str, float]:
    out = {}
    for n, p in model.named_parameters():
        g = getattr(p, "main_grad", None)
        if g is None:
            g = p.grad
        if g is not None:
            out[n] = float(g.float().norm())
    return out


def save_spike_snapshot(root: str | Path, step: int, grad_norm: float, train_engine: Any, batch: Any, cfg: GradSpikeDebugConfig,
                        trainer_state: dict | None = None) -> Path:
    from axrl_b200.train.checkpoint import save_dist_checkpoint

    root = Path(root) / "spike_snapshots"
    d = save_dist_checkpoint(root, step, train_engine.model, train_engine.optim, most_recent_k=None)
    torch.save({k: v.cpu() for k, v in batch.tensors.items()}, d / "batch_rank0.pt")
    if cfg.save_per_param_grads:
        torch.save(per_param_grad_norms(train_engine.model), d / "grad_info_rank0.pt")
    torch.save(trainer_state or {}, d / "trainer.pt")
    (d / "axrl_metadata.json").write_text(json.dumps({"step": step, "grad_norm": grad_norm, "spike_ratio": cfg.spike_ratio}))
    snaps = sorted(p for p in root.glob("iter_*") if p.is_dir())
    for old in snaps[: -cfg.max_snapshots]:
        shutil.rmtree(old, ignore_errors=True)
    return d


def replay_snapshot(snapshot_dir: str | Path, train_engine: Any, trainer: Any) -> dict:
    """Reload weights + optimizer + batch of a snapshot and recompute the gradient (no update)."""
    from axrl_b200.data.sample import SampleBatch
    from axrl_b200.train.checkpoint import load_dist_checkpoint

    d = Path(snapshot_dir)
    load_dist_checkpoint(d.parent, train_engine.model, train_engine.optim, step=int(d.name.split("_")[1]))
    tensors = torch.load(d / "batch_rank0.pt")
    batch = SampleBatch(tensors)
    meta = json.loads((d / "axrl_metadata.json").read_text())
    opt = train_engine.optim
    saved = (opt.master.clone(), opt.exp_avg.clone(), opt.exp_avg_sq.clone(), opt.step_count)
    m = train_engine.train_step(batch, trainer)
    opt.master.copy_(saved[0]), opt.exp_avg.copy_(saved[1]), opt.exp_avg_sq.copy_(saved[2])
    opt.step_count = saved[3]
    opt.bf16.copy_(opt.master)
    return {"recorded_grad_norm": meta["grad_norm"], "replayed_grad_norm": m["grad_norm"]}

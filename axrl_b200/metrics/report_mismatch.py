"""Training-vs-inference mismatch report.

Reference: ``report_mismatch`` (``axrl/metrics/report_mismatch.py``) run by the ``mismatch_test``
mode (``axrl/pipeline/controller.py:1693-1779``): after rollouts, the trainer recomputes the
log-probs of every sampled token; the report measures how far the rollout engine's log-probs are
from the trainer's (and optionally compares against a baseline run's samples), lists the most
mismatched tokens, and draws the distribution.  The figure is written as a self-contained SVG.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np
import torch


@dataclass
class MismatchReportTask:
    exp_name: str
    exp_sample_data_path: str
    baseline_sample_data_path: str | None = None
    baseline_name: str = "baseline"
    output_fig_path: str | None = None
    output_txt_path: str | None = None
    model: Any = None
    top_k: int = 50


@dataclass
class MCoreRunMetrics:
    end_to_end_time_sec: float = 0.0
    old_logprobs_gpu_usage: list = field(default_factory=list)


@dataclass
class MismatchRunResult:
    success: bool
    grpo_config: Any = None
    metadata: dict = field(default_factory=dict)
    response_metrics: dict = field(default_factory=dict)
    rollout_throughput: float | None = None
    mcore: MCoreRunMetrics | None = None
    mismatch_metrics: dict = field(default_factory=dict)


def mismatch_metrics(batch: Any, prefix: str = "mismatch") -> dict[str, float]:
    """Statistics of ``old_logprobs - rollout_logprobs`` over trained tokens."""
    mask = batch["loss_mask"].bool()
    d = (batch["old_logprobs"] - batch["rollout_logprobs"])[mask].double()
    if d.numel() == 0:
        return {f"{prefix}/num_tokens": 0.0}
    r = torch.exp(d.clamp(-20, 20))
    k3 = (torch.exp(-d) - 1 + d).mean()  # KL(rollout || train) estimate with samples from rollout
    q = torch.quantile(d.abs().float(), torch.tensor([0.5, 0.9, 0.99, 0.999]))
    out = {
        f"{prefix}/num_tokens": float(d.numel()),
        f"{prefix}/abs_diff_mean": float(d.abs().mean()),
        f"{prefix}/abs_diff_max": float(d.abs().max()),
        f"{prefix}/abs_diff_p50": float(q[0]), f"{prefix}/abs_diff_p90": float(q[1]),
        f"{prefix}/abs_diff_p99": float(q[2]), f"{prefix}/abs_diff_p999": float(q[3]),
        f"{prefix}/kl_k3": float(k3),
        f"{prefix}/ratio_mean": float(r.mean()),
        f"{prefix}/ratio_min": float(r.min()), f"{prefix}/ratio_max": float(r.max()),
        f"{prefix}/frac_ratio_outside_0.8_1.25": float(((r < 0.8) | (r > 1.25)).double().mean()),
    }
    if "ref_logprobs" in batch.tensors:
        dr = (batch["old_logprobs"] - batch["ref_logprobs"])[mask].double()
        out[f"{prefix}/policy_drift_abs_mean"] = float(dr.abs().mean())
    return out


def top_mismatched_tokens(batch: Any, k: int = 50) -> list[tuple[int, int, int, float, float]]:
    """(row, position, token, rollout lp, trainer lp) of the ``k`` largest |differences|."""
    mask = batch["loss_mask"].bool()
    d = (batch["old_logprobs"] - batch["rollout_logprobs"]).abs().masked_fill(~mask, -1.0)
    flat = d.reshape(-1)
    k = min(k, int(mask.sum()))
    if k <= 0:
        return []
    idx = torch.topk(flat, k).indices
    S = d.shape[1]
    out = []
    for i in idx.tolist():
        r, c = divmod(i, S)
        out.append((r, c, int(batch["labels"][r, c]), float(batch["rollout_logprobs"][r, c]), float(batch["old_logprobs"][r, c])))
    return out


def _svg_histogram(series: dict[str, np.ndarray], path: str, bins: int = 60) -> None:
    W, H, pad = 720, 360, 40
    allv = np.concatenate([v for v in series.values() if v.size]) if series else np.zeros(1)
    lo, hi = float(np.log10(max(allv.min(), 1e-8))), float(np.log10(max(allv.max(), 1e-7)))
    hi = max(hi, lo + 1e-3)
    edges = np.linspace(lo, hi, bins + 1)
    colors = ["#1f77b4", "#d62728", "#2ca02c"]
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}">',
             f'<text x="{pad}" y="20" font-size="14">|old_logprob - rollout_logprob| (log10), per trained token</text>']
    peak = 1
    hists = {}
    for name, v in series.items():
        h, _ = np.histogram(np.log10(np.maximum(v, 1e-8)), bins=edges)
        hists[name] = h
        peak = max(peak, int(h.max()))
    for j, (name, h) in enumerate(hists.items()):
        pts = " ".join(f"{pad + (W - 2 * pad) * i / bins:.1f},{H - pad - (H - 2 * pad) * c / peak:.1f}" for i, c in enumerate(h))
        parts.append(f'<polyline fill="none" stroke="{colors[j % 3]}" stroke-width="2" points="{pts}"/>')
        parts.append(f'<text x="{W - 200}" y="{40 + 16 * j}" fill="{colors[j % 3]}" font-size="12">{name}</text>')
    parts.append(f'<text x="{pad}" y="{H - 10}" font-size="11">10^{lo:.1f}</text><text x="{W - pad - 40}" y="{H - 10}" font-size="11">10^{hi:.1f}</text>')
    parts.append("</svg>")
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text("\n".join(parts))


def report_mismatch(task: MismatchReportTask, metric_logger: Any = None, step: int = 0) -> dict[str, float]:
    from axrl_b200.utils.zst_utils import load_zst

    exp = load_zst(task.exp_sample_data_path)
    metrics = mismatch_metrics(exp, f"mismatch/{task.exp_name}")
    series = {task.exp_name: (exp["old_logprobs"] - exp["rollout_logprobs"])[exp["loss_mask"].bool()].abs().numpy()}
    if task.baseline_sample_data_path is not None:
        base = load_zst(task.baseline_sample_data_path)
        bm = mismatch_metrics(base, f"mismatch/{task.baseline_name}")
        metrics.update(bm)
        a, b = metrics[f"mismatch/{task.exp_name}/kl_k3"], bm[f"mismatch/{task.baseline_name}/kl_k3"]
        metrics["mismatch/kl_k3_ratio_vs_baseline"] = a / b if b > 0 else math.inf
        series[task.baseline_name] = (base["old_logprobs"] - base["rollout_logprobs"])[base["loss_mask"].bool()].abs().numpy()
    if task.output_txt_path:
        Path(task.output_txt_path).parent.mkdir(parents=True, exist_ok=True)
        lines = [f"# top {task.top_k} mismatched tokens of {task.exp_name}: row pos token rollout_lp trainer_lp |diff|"]
        for r, c, t, a, b in top_mismatched_tokens(exp, task.top_k):
            lines.append(f"{r}\t{c}\t{t}\t{a:.5f}\t{b:.5f}\t{abs(a - b):.5f}")
        Path(task.output_txt_path).write_text("\n".join(lines) + "\n")
    if task.output_fig_path:
        _svg_histogram(series, str(Path(task.output_fig_path).with_suffix(".svg")))
    if metric_logger is not None:
        metric_logger.log_scalars(metrics, step=step)
    return metrics

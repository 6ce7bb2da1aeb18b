"""Per-response metrics and their aggregation (reference ``axrl/metrics/response_metric.py:15-231``).

A :class:`ResponseMetric` describes one generated response:

* size and diversity: ``token_count`` (== ``response_length``), ``token_unique_ratio``, the longest
  word and line in characters, and ``ngram_repetition`` — the share of 20-token n-grams that occur
  more than once, computed over 4000-token chunks and weighted by chunk length, so degenerate loops
  are caught without quadratic memory;
* reasoning-behaviour cues: 1.0 when the lower-cased text contains a backtracking, verification or
  causal cue phrase (the cue lists are the metric's definition and follow the reference so the
  dashboards compare);
* rollout bookkeeping: cached tokens, retries (partial-rollout resumptions), end-to-end seconds and
  one 0/1 counter per finish reason;
* ``is_low_quality``: long and highly repetitive, or one enormous line with repetition.

:func:`aggregate_response_metrics` averages every numeric field over all responses and separately
over positively and non-positively scored ones (``__all`` / ``__pos`` / ``__neg`` suffixes), and
:func:`aggregate_response_metrics_by_subset` does the same per ``conversation.extra[subset_key]``.
"""

from __future__ import annotations

from collections import Counter, defaultdict
from dataclasses import asdict, dataclass, field
from typing import Any, Sequence

import numpy as np

FINISH_REASONS = ("stop", "length", "tool_calls", "function_call", "content_filter", "abort")

CUES: dict[str, tuple[str, ...]] = {
    "backtracking": ("wait", "second thought", "re-examine", "rethink", "reconsider", "start over", "try another", "backtrack"),
    "verification": ("check", "verify", "confirm", "ensure", "validate", "cross-check"),
    "causal": ("because", "leads to", "due to", "consequence", "since", "therefore", "thus"),
}


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
    repetition_ratio: float = 0.0  # share of repeated 4-grams (cheap, always filled)
    token_unique_ratio: float = 0.0
    word_length_max: int = 0
    line_length_max: int = 0
    ngram_repetition: float = 0.0
    reasoning_behavior_backtracking: float = 0.0
    reasoning_behavior_verification: float = 0.0
    reasoning_behavior_causal: float = 0.0
    rollout_cached_tokens: int = 0
    rollout_num_retry: int = 0
    is_low_quality: float | None = None
    extra: dict = field(default_factory=dict)

    @property
    def token_count(self) -> int:
        return self.response_length

    @staticmethod
    def repetition(tokens: Sequence[int], n: int = 4) -> float:
        if len(tokens) < n + 1:
            return 0.0
        grams = [tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1)]
        return 1.0 - len(set(grams)) / len(grams)

    def to_dict(self) -> dict[str, float]:
        """Numeric fields, finish-reason counters and numeric ``extra`` entries, flat."""
        d = {k: v for k, v in asdict(self).items() if k not in ("extra", "finish_reason")}
        d["token_count"] = self.response_length
        for r in FINISH_REASONS:
            d[f"rollout_finish_reason_{r}"] = 1.0 if self.finish_reason == r else 0.0
        d.update({k: v for k, v in self.extra.items() if isinstance(v, (int, float, bool))})
        return {k: (float("nan") if v is None else float(v)) for k, v in d.items()}


def ngram_repetition(tokens: Sequence[int], n: int = 20, chunk: int = 4000) -> float:
    """Length-weighted share of n-grams (per ``chunk``-token piece) that occur more than once."""
    if len(tokens) < n:
        return 0.0
    reps, weights = [], []
    for s in range(0, len(tokens), chunk):
        piece = tuple(tokens[s:s + chunk])
        counts = Counter(piece[i:i + n] for i in range(len(piece) - n + 1))
        total = sum(counts.values())
        reps.append(sum(c for c in counts.values() if c > 1) / total if total else 0.0)
        weights.append(len(piece))
    return float(np.average(reps, weights=weights))


def low_quality(m: ResponseMetric) -> bool:
    if m.response_length >= 4096 and m.ngram_repetition >= 0.4 and m.token_unique_ratio <= 0.1:
        return True
    return m.line_length_max >= 8192 and m.ngram_repetition >= 0.2


class ResponseMetricCalculator:
    """GenerationOutput (ids, text, rollout bookkeeping) -> :class:`ResponseMetric`."""

    def __init__(self, config: Any = None) -> None:
        self.config = config

    def process(self, out: Any, prompt_length: int = 0, score: float | None = None) -> ResponseMetric:
        tokens = [int(t) for t in np.asarray(out.output_ids).reshape(-1)]
        text = getattr(out, "output_text", "") or ""
        lower = text.lower()
        words = text.split()
        lines = [ln for ln in text.splitlines() if ln.strip()]
        m = ResponseMetric(
            score=score, response_length=len(tokens), prompt_length=prompt_length,
            finish_reason=str(getattr(out, "finish_reason", "stop") or "stop"),
            elapsed_seconds=float(getattr(out, "e2e_elapsed_seconds", 0.0) or 0.0),
            repetition_ratio=ResponseMetric.repetition(tokens),
            token_unique_ratio=len(set(tokens)) / max(1, len(tokens)),
            word_length_max=max((len(w) for w in words), default=0),
            line_length_max=max((len(ln) for ln in lines), default=0),
            ngram_repetition=ngram_repetition(tokens),
            reasoning_behavior_backtracking=float(any(c in lower for c in CUES["backtracking"])),
            reasoning_behavior_verification=float(any(c in lower for c in CUES["verification"])),
            reasoning_behavior_causal=float(any(c in lower for c in CUES["causal"])),
            rollout_cached_tokens=int(getattr(out, "cached_tokens", 0) or 0),
            rollout_num_retry=int(getattr(out, "retry", 0) or 0),
        )
        m.is_low_quality = float(low_quality(m))
        return m

    async def generate(self, out: Any) -> ResponseMetric:
        return self.process(out)


def _mean_table(rows: list[dict[str, float]]) -> dict[str, float]:
    keys = sorted({k for r in rows for k in r})
    out = {}
    for k in keys:
        vals = np.asarray([r.get(k, np.nan) for r in rows], dtype=np.float64)
        vals = vals[~np.isnan(vals)]
        if vals.size:
            out[k] = float(vals.mean())
    return out


def aggregate_response_metrics(metrics: Sequence[ResponseMetric], prefix: str = "All-Rollouts", wall_seconds: float | None = None,
                               *, total_seconds: float | None = None) -> dict[str, float]:
    """Means over all / positively scored / non-positively scored responses, plus the summary keys
    ``{prefix}/num``, ``response_length_{mean,max,min}``, ``score_{mean,std}``, ``finish_<r>_ratio``
    and ``throughput_tokens_per_second`` (response tokens over ``wall_seconds``)."""
    if not metrics:
        return {}
    wall_seconds = wall_seconds if wall_seconds is not None else total_seconds
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
    splits = {"all": list(metrics), "pos": [m for m in metrics if m.score is not None and m.score > 0],
              "neg": [m for m in metrics if m.score is not None and m.score <= 0]}
    for tag, ms in splits.items():
        if not ms:
            continue
        rows = [m.to_dict() for m in ms]
        for k, v in _mean_table(rows).items():
            out[f"{prefix}/{k}__{tag}"] = v
        counts = [m.response_length for m in ms]
        out[f"{prefix}/rollout_number__{tag}"] = float(len(ms))
        out[f"{prefix}/token_count_max__{tag}"] = float(max(counts))
        out[f"{prefix}/token_count_min__{tag}"] = float(min(counts))
    if wall_seconds:
        out[f"{prefix}/throughput_tokens_per_second"] = float(lens.sum() / wall_seconds)
    return out


def aggregate_response_metrics_by_subset(results: Sequence[Any], subset_key: str, prefix: str) -> dict[str, float]:
    """Per-subset aggregation keyed by ``result.conversation.extra[subset_key]``; empty when fewer
    than two subsets are present (a single subset repeats the overall numbers)."""
    groups: dict[str, list[ResponseMetric]] = defaultdict(list)
    for r in results:
        conv = getattr(r, "conversation", None)
        val = conv.extra.get(subset_key) if conv is not None and getattr(conv, "extra", None) else None
        if val is not None:
            groups[str(val)].append(r.metric)
    if len(groups) <= 1:
        return {}
    out: dict[str, float] = {}
    for name, ms in sorted(groups.items()):
        out.update(aggregate_response_metrics(ms, f"{prefix}/{name}"))
    return out

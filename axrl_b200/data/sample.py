"""Per-sample training record and its batched tensor form.

``Sample`` carries the same fields as reference ``axrl/data/sample.py:22-69``
(left-shifted labels, loss mask, rollout/old/ref/teacher logprobs, values,
returns, turn ids and rewards, routing handles, prefix-merge info,
trajectory id).  ``SampleBatch`` replaces the reference's TensorDict: a plain
``dict[str, Tensor]`` with a row count plus per-row Python objects, which is
all the trainer needs and keeps the host data plane dependency-free.

Padding rows (``index == -1``, zero loss mask) make a global batch divisible
by the DP size (reference ``axrl/data/global_batch_iterator.py:100-117``).
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields
from typing import Any, Sequence

import numpy as np
import torch

from axrl_b200.configs import IGNORE_INDEX

_I32 = ("input_ids", "labels", "position_ids", "turn_index")
_F32 = ("advantage", "rollout_logprobs", "old_logprobs", "ref_logprobs", "teacher_logprobs", "old_values", "returns", "turn_reward")
_BOOL = ("loss_mask", "attention_mask")
_OBJ = ("merge_info", "routing_handles_per_path")


def _as(arr: Any, dtype: Any) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(arr), dtype=dtype)


@dataclass
class Sample:
    input_ids: np.ndarray
    labels: np.ndarray
    loss_mask: np.ndarray
    attention_mask: np.ndarray
    position_ids: np.ndarray
    reward: float
    reward_baseline: float
    advantage: np.ndarray
    rollout_logprobs: np.ndarray | None = None
    old_logprobs: np.ndarray | None = None
    ref_logprobs: np.ndarray | None = None
    teacher_logprobs: np.ndarray | None = None
    old_values: np.ndarray | None = None
    returns: np.ndarray | None = None
    turn_index: np.ndarray | None = None
    turn_reward: np.ndarray | None = None
    routing_handles_per_path: list | None = None
    merge_info: Any = None
    trajectory_id: int = -1

    def __post_init__(self) -> None:
        for name in _I32:
            v = getattr(self, name)
            if v is not None:
                setattr(self, name, _as(v, np.int32))
        for name in _F32:
            v = getattr(self, name)
            if v is not None:
                setattr(self, name, _as(v, np.float32))
        for name in _BOOL:
            setattr(self, name, _as(getattr(self, name), np.bool_))

    def __len__(self) -> int:
        return int(self.input_ids.shape[0])

    @staticmethod
    def from_tokens(
        prompt_ids: Sequence[int],
        response_ids: Sequence[int],
        *,
        reward: float = 0.0,
        advantage: float = 0.0,
        rollout_logprobs: Sequence[float] | None = None,
        trajectory_id: int = -1,
    ) -> "Sample":
        """Build a single-turn sample: labels are input_ids shifted left by one;
        the loss mask covers exactly the positions whose label is a response token."""
        ids = list(prompt_ids) + list(response_ids)
        n, p = len(ids), len(prompt_ids)
        labels = ids[1:] + [IGNORE_INDEX]
        loss_mask = np.zeros(n, dtype=bool)
        loss_mask[p - 1 : n - 1] = True
        lp = None
        if rollout_logprobs is not None:
            lp = np.zeros(n, dtype=np.float32)
            lp[p - 1 : n - 1] = np.asarray(rollout_logprobs, dtype=np.float32)
        return Sample(
            input_ids=np.asarray(ids),
            labels=np.asarray(labels),
            loss_mask=loss_mask,
            attention_mask=np.ones(n, dtype=bool),
            position_ids=np.arange(n),
            reward=float(reward),
            reward_baseline=0.0,
            advantage=np.where(loss_mask, advantage, 0.0).astype(np.float32),
            rollout_logprobs=lp,
            trajectory_id=trajectory_id,
        )


def get_prompt_ids(sample: Sample) -> list[int]:
    """Tokens before the first trainable label position (inclusive of that position)."""
    idx = np.flatnonzero(sample.loss_mask)
    end = int(idx[0]) + 1 if idx.size else len(sample)
    return sample.input_ids[:end].tolist()


def get_response_ids(sample: Sample) -> list[int]:
    idx = np.flatnonzero(sample.loss_mask)
    return [] if not idx.size else sample.labels[idx].tolist()


class SampleBatch:
    """Row-major batch: ``tensors[key]`` has leading dim ``n_rows``; ``objects[key]``
    is a per-row Python list (merge info, routing handles)."""

    def __init__(self, tensors: dict[str, torch.Tensor], objects: dict[str, list] | None = None, n_rows: int | None = None):
        self.tensors = tensors
        self.objects = objects or {}
        if n_rows is None:
            n_rows = next(iter(tensors.values())).shape[0] if tensors else 0
        self.n_rows = int(n_rows)

    def __len__(self) -> int:
        return self.n_rows

    def __getitem__(self, key: str) -> torch.Tensor:
        return self.tensors[key]

    def __setitem__(self, key: str, value: torch.Tensor) -> None:
        assert value.shape[0] == self.n_rows, f"{key}: {value.shape[0]} rows != {self.n_rows}"
        self.tensors[key] = value

    def __contains__(self, key: str) -> bool:
        return key in self.tensors or key in self.objects

    def get(self, key: str, default: Any = None) -> Any:
        if key in self.tensors:
            return self.tensors[key]
        return self.objects.get(key, default)

    def keys(self) -> list[str]:
        return list(self.tensors) + list(self.objects)

    def to(self, device: Any, non_blocking: bool = False) -> "SampleBatch":
        return SampleBatch({k: v.to(device, non_blocking=non_blocking) for k, v in self.tensors.items()}, dict(self.objects), self.n_rows)

    def select_rows(self, rows: Sequence[int]) -> "SampleBatch":
        idx = torch.as_tensor(list(rows), dtype=torch.long)
        tensors = {k: v.index_select(0, idx.to(v.device)) for k, v in self.tensors.items()}
        objects = {k: [v[i] for i in rows] for k, v in self.objects.items()}
        return SampleBatch(tensors, objects, len(rows))

    @staticmethod
    def concat(batches: Sequence["SampleBatch"]) -> "SampleBatch":
        batches = [b for b in batches if len(b)]
        assert batches, "nothing to concatenate"
        width = max(b.tensors["input_ids"].shape[1] for b in batches)
        tensors: dict[str, torch.Tensor] = {}
        for k in batches[0].tensors:
            parts = []
            for b in batches:
                t = b.tensors[k]
                if t.dim() >= 2 and t.shape[1] < width:
                    pad = torch.zeros((t.shape[0], width - t.shape[1], *t.shape[2:]), dtype=t.dtype, device=t.device)
                    if k == "labels":
                        pad.fill_(IGNORE_INDEX)
                    t = torch.cat([t, pad], 1)
                parts.append(t)
            tensors[k] = torch.cat(parts, 0)
        objects = {k: sum((b.objects.get(k, [None] * len(b)) for b in batches), []) for k in batches[0].objects}
        return SampleBatch(tensors, objects, sum(len(b) for b in batches))

    @staticmethod
    def from_samples(samples: Sequence[Sample], *, max_length: int | None = None) -> "SampleBatch":
        return tensorize_samples(samples, max_length=max_length)


# Compatibility alias for code written against the reference's name.
SampleTensorDict = SampleBatch


def tensorize_samples(samples: Sequence[Sample], *, max_length: int | None = None) -> SampleBatch:
    """Right-pad a list of samples into (B, T) tensors."""
    assert samples, "empty sample list"
    T = max(len(s) for s in samples) if max_length is None else max_length
    B = len(samples)
    out: dict[str, torch.Tensor] = {}
    spec = [(n, torch.int32, 0) for n in _I32] + [(n, torch.float32, 0.0) for n in _F32] + [(n, torch.bool, False) for n in _BOOL]
    for name, dtype, fill in spec:
        vals = [getattr(s, name) for s in samples]
        if all(v is None for v in vals):
            if name in ("turn_index",):
                continue
            if name in ("teacher_logprobs", "old_values", "returns", "turn_reward"):
                continue
        buf = torch.full((B, T), IGNORE_INDEX if name == "labels" else fill, dtype=dtype)
        for i, v in enumerate(vals):
            if v is None:
                continue
            n = min(len(v), T)
            buf[i, :n] = torch.from_numpy(np.asarray(v[:n]))
        out[name] = buf
    out["reward"] = torch.tensor([s.reward for s in samples], dtype=torch.float32)
    out["reward_baseline"] = torch.tensor([s.reward_baseline for s in samples], dtype=torch.float32)
    out["trajectory_id"] = torch.tensor([s.trajectory_id for s in samples], dtype=torch.int64)
    out["index"] = torch.arange(B, dtype=torch.int64)
    out["seq_len"] = torch.tensor([int(s.attention_mask.sum()) for s in samples], dtype=torch.int32)
    objects = {k: [getattr(s, k) for s in samples] for k in _OBJ}
    return SampleBatch(out, objects, B)


def samples_from_batch(batch: SampleBatch) -> list[Sample]:
    """Inverse of :func:`tensorize_samples` (drops right padding per row)."""
    res = []
    names = {f.name for f in fields(Sample)}
    for i in range(len(batch)):
        n = int(batch["seq_len"][i]) if "seq_len" in batch.tensors else int(batch["attention_mask"][i].sum())
        kw: dict[str, Any] = {}
        for k, v in batch.tensors.items():
            if k in names and v.dim() == 2:
                kw[k] = v[i, :n].numpy()
        kw["reward"] = float(batch["reward"][i])
        kw["reward_baseline"] = float(batch["reward_baseline"][i])
        kw["trajectory_id"] = int(batch["trajectory_id"][i])
        for k in _OBJ:
            kw[k] = batch.objects.get(k, [None] * len(batch))[i]
        res.append(Sample(**kw))
    return res


def make_padding_samples(count: int, length: int, pad_token_id: int = 0) -> list[Sample]:
    """Zero-loss filler rows used to round a global batch up to a DP multiple."""
    out = []
    for _ in range(count):
        out.append(
            Sample(
                input_ids=np.full(length, pad_token_id),
                labels=np.full(length, IGNORE_INDEX),
                loss_mask=np.zeros(length, dtype=bool),
                attention_mask=np.ones(length, dtype=bool),
                position_ids=np.arange(length),
                reward=0.0,
                reward_baseline=0.0,
                advantage=np.zeros(length, dtype=np.float32),
                rollout_logprobs=np.zeros(length, dtype=np.float32),
                trajectory_id=-1,
            )
        )
    return out

"""Packed micro-batches and token-balanced micro-batch splitting.

Reference counterparts:
* THD packing (remove padding, cu_seqlens) – ``axrl/utils/megatron/pack_utils.py:26-119``;
* prefix-tree forest packing for merged samples – ``axrl/utils/megatron/magi_forward.py:890-1054``;
* Karmarkar–Karp token balancing with a DP-wide micro-batch count –
  ``axrl/utils/megatron/seqlen_balancing.py:259-342``.

A micro-batch is one flat token stream: per-row valid tokens concatenated,
with an :class:`AttnSpec` describing who attends to whom (one causal triple per
flat row; the per-node ranges of the trie for merged rows, shifted to the row's
offset).  The packed layout is what every kernel consumes; no padding is
materialised.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np
import torch

from axrl_b200.configs import IGNORE_INDEX
from axrl_b200.data.sample import SampleBatch
from axrl_b200.ops.attention_spec import AttnSpec, spec_from_triples

TOKEN_KEYS_F32 = ("advantage", "rollout_logprobs", "old_logprobs", "ref_logprobs", "teacher_logprobs", "old_values", "returns", "turn_reward")


@dataclass
class PackedMicroBatch:
    rows: list[int]  # batch row indices in this micro-batch
    row_len: list[int]  # valid tokens per row
    row_off: list[int]  # offset of each row in the packed stream
    ids: torch.Tensor  # (T,) int64
    pos: torch.Tensor  # (T,) int32
    labels: torch.Tensor  # (T,) int64 (IGNORE for non-trainable)
    loss_mask: torch.Tensor  # (T,) bool
    token_row: torch.Tensor  # (T,) int64 local row index (0..len(rows)-1)
    spec: AttnSpec
    fields: dict[str, torch.Tensor]  # per-token float fields (advantage, logprobs, ...)
    merge_info: list | None = None
    token_col: torch.Tensor | None = None  # (T,) column of each token in its row when rows are not contiguous (CP)

    @property
    def num_tokens(self) -> int:
        return int(self.ids.numel())

    def to(self, device, non_blocking: bool = True) -> "PackedMicroBatch":  # noqa: ANN001
        from axrl_b200.utils import iostats

        if torch.device(device).type == "cuda":
            iostats.add_h2d(self.ids, self.pos, self.labels, self.loss_mask, self.token_row, *self.fields.values())
        mv = lambda t: t.to(device, non_blocking=non_blocking)  # noqa: E731
        return PackedMicroBatch(self.rows, self.row_len, self.row_off, mv(self.ids), mv(self.pos), mv(self.labels), mv(self.loss_mask),
                                mv(self.token_row), self.spec.to(device), {k: mv(v) for k, v in self.fields.items()}, self.merge_info,
                                None if self.token_col is None else mv(self.token_col))

    def unpack(self, flat: torch.Tensor, width: int) -> torch.Tensor:
        """(T,) per-token values -> (rows, width) right-padded with zeros."""
        out = torch.zeros((len(self.rows), width), dtype=flat.dtype, device=flat.device)
        if self.token_col is not None:
            keep = self.token_row >= 0
            out[self.token_row[keep], self.token_col[keep]] = flat[keep]
            return out
        n = sum(self.row_len)  # trailing padding tokens (token_row -1) are dropped
        trow = self.token_row[:n]
        col = torch.arange(n, device=flat.device) - torch.as_tensor(self.row_off, device=flat.device)[trow]
        out[trow, col] = flat[:n]
        return out


def _row_valid(batch: SampleBatch, r: int) -> int:
    return int(batch["seq_len"][r]) if "seq_len" in batch.tensors else int(batch["attention_mask"][r].sum())


def pack_rows(batch: SampleBatch, rows: list[int], pad_to: int = 1) -> PackedMicroBatch:
    """Flatten ``rows`` of a right-padded batch into one packed stream (host tensors).

    ``pad_to`` rounds the stream length up (e.g. to a multiple of the TP size for sequence
    parallelism) with a trailing causal segment of untrained padding tokens."""
    ids, pos, lab, lm, trow = [], [], [], [], []
    fields = {k: [] for k in TOKEN_KEYS_F32 if k in batch.tensors}
    triples = []
    infos = batch.objects.get("merge_info") or [None] * len(batch)
    row_len, row_off = [], []
    off = 0
    for li, r in enumerate(rows):
        n = _row_valid(batch, r)
        info = infos[r]
        if info is not None:
            n = info.total_padded
            for (q0, q1), (k0, k1), t in zip(info.q_ranges, info.k_ranges, info.attn_type_map):
                triples.append((q0 + off, q1 + off, k0 + off, k1 + off, int(t)))
        else:
            triples.append((off, off + n, off, off + n, 1))
        ids.append(batch["input_ids"][r, :n])
        pos.append(batch["position_ids"][r, :n])
        lab.append(batch["labels"][r, :n])
        lm.append(batch["loss_mask"][r, :n])
        for k in fields:
            fields[k].append(batch[k][r, :n])
        trow.append(torch.full((n,), li, dtype=torch.int64))
        row_len.append(n)
        row_off.append(off)
        off += n
    pad = (-off) % max(1, pad_to)
    if pad:
        triples.append((off, off + pad, off, off + pad, 1))
        ids.append(torch.zeros(pad, dtype=torch.int64))
        pos.append(torch.arange(pad, dtype=torch.int64))
        lab.append(torch.full((pad,), IGNORE_INDEX, dtype=torch.int64))
        lm.append(torch.zeros(pad, dtype=torch.bool))
        for k in fields:
            fields[k].append(torch.zeros(pad, dtype=batch[k].dtype))
        trow.append(torch.full((pad,), -1, dtype=torch.int64))
        off += pad
    spec = spec_from_triples(triples, off)
    return PackedMicroBatch(
        rows=list(rows), row_len=row_len, row_off=row_off,
        ids=torch.cat(ids).long(), pos=torch.cat(pos).int(), labels=torch.cat(lab).long(), loss_mask=torch.cat(lm).bool(),
        token_row=torch.cat(trow), spec=spec, fields={k: torch.cat(v).float() for k, v in fields.items()},
        merge_info=[infos[r] for r in rows] if any(infos[r] is not None for r in rows) else None,
    )


def karmarkar_karp(lengths: list[int], k: int) -> list[list[int]]:
    """Largest-differencing partition of item indices into ``k`` bins of near-equal sum."""
    if k <= 1:
        return [list(range(len(lengths)))]
    heap = []
    for i, w in enumerate(lengths):
        parts = [(0, []) for _ in range(k - 1)] + [(w, [i])]
        parts.sort(key=lambda x: x[0], reverse=True)
        spread = parts[0][0] - parts[-1][0]
        heapq.heappush(heap, (-spread, i, parts))
    while len(heap) > 1:
        _, i1, a = heapq.heappop(heap)
        _, _, b = heapq.heappop(heap)
        # combine largest of a with smallest of b, etc.
        merged = [(a[j][0] + b[k - 1 - j][0], a[j][1] + b[k - 1 - j][1]) for j in range(k)]
        merged.sort(key=lambda x: x[0], reverse=True)
        heapq.heappush(heap, (-(merged[0][0] - merged[-1][0]), i1, merged))
    return [sorted(p[1]) for p in heap[0][2]]


def split_balanced(lengths: list[int], max_tokens: int, min_count: int = 1, multiple_of: int = 1) -> list[list[int]]:
    """Token-balanced micro-batches with at most ``max_tokens`` each (a single longer row
    gets its own micro-batch).  The count is raised to ``min_count`` (e.g. the DP-wide max)
    and rounded up to ``multiple_of`` (pipeline virtual stages)."""
    if not lengths:
        return []
    total = sum(lengths)
    k = max(min_count, -(-total // max_tokens), 1)
    k = min(k, len(lengths)) if min_count <= len(lengths) else k
    while True:
        k = -(-k // multiple_of) * multiple_of
        parts = karmarkar_karp(lengths, k) if k <= len(lengths) else [[i] for i in range(len(lengths))] + [[] for _ in range(k - len(lengths))]
        worst = max(sum(lengths[i] for i in p) for p in parts)
        if worst <= max_tokens or k >= len(lengths):
            break
        k += 1
    # longest first (sum of squared lengths ~ attention cost), empty bins last
    parts.sort(key=lambda p: -sum(lengths[i] ** 2 for i in p))
    return parts


def num_micro_batches_for(lengths: list[int], max_tokens: int) -> int:
    return len(split_balanced(lengths, max_tokens))

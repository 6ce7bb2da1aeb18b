"""Range-list attention specification shared by the varlen and tree paths.

An attention problem over a packed token buffer is a list of *triples*
``(q_range, k_range, type)``: queries in ``[q0, q1)`` attend to keys in
``[k0, k1)`` either fully (type 0) or causally (type 1: key ``k0 + j`` is
visible to query ``q0 + i`` iff ``j <= i``).  This is the same vocabulary as
the reference's MagiAttention calls (``axrl/utils/megatron/magi_forward.py:445-466``)
and covers flat causal packing (one causal triple per sequence), prefix trees
(full to ancestors + causal to self) and CP-local shards.

The kernels want two groupings of the triples:

* by query range (forward and dQ): each q-segment owns a contiguous run of
  k-ranges, processed with one online softmax;
* by key range (dK/dV): each k-segment owns a run of q-ranges.

Both are built once per micro-batch on the host as int32 tables and copied to
the device with one H2D each.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch


@dataclass
class AttnSpec:
    # grouped by q: qseg[i] = (q0, q1, first, last) into kr (k0, k1, type)
    qseg: torch.Tensor  # (Nq, 4) int32
    kr: torch.Tensor  # (Nk_items, 3) int32
    # grouped by k: kseg[j] = (k0, k1, first, last) into qr (q0, q1, type)
    kseg: torch.Tensor  # (Nk, 4) int32
    qr: torch.Tensor  # (Nq_items, 3) int32
    total_q: int
    total_k: int
    max_q_len: int
    max_k_len: int
    # (segment index, tile start) work tables for the forward (128-row q tiles) and
    # backward (64-row k tiles) kernels.
    fwd_tiles: torch.Tensor | None = None
    bwd_tiles: torch.Tensor | None = None
    bwd_tiles_tc: torch.Tensor | None = None  # 128-key tiles of the tcgen05 backward
    # host-side token layout for sequence mixers that need whole sequences (Gated DeltaNet under
    # context parallelism: see ``parallel.context_parallel.CPSeqLayout``); None = flat packing
    seq_layout: Any = None
    # context parallelism: one spec per key source rank, queries local and keys in that rank's
    # own stream coordinates (ring attention attends to each source's chunk as it arrives)
    cp_sources: list | None = None

    def to(self, device, non_blocking: bool = True) -> "AttnSpec":  # noqa: ANN001
        """Move every table to ``device`` in ONE host->device copy (pinned staging)."""
        parts = [self.qseg, self.kr, self.kseg, self.qr, self.fwd_tiles, self.bwd_tiles, self.bwd_tiles_tc]
        flat = torch.cat([p.reshape(-1) for p in parts])
        if torch.device(device).type == "cuda":
            flat = flat.pin_memory().to(device, non_blocking=non_blocking)
        out, off = [], 0
        for p in parts:
            n = p.numel()
            out.append(flat[off:off + n].view(p.shape))
            off += n
        srcs = [c.to(device, non_blocking) for c in self.cp_sources] if self.cp_sources is not None else None
        return AttnSpec(*out[:4], self.total_q, self.total_k, self.max_q_len, self.max_k_len, out[4], out[5], out[6], self.seq_layout,
                        srcs)

    def triples(self) -> list[tuple[int, int, int, int, int]]:
        out = []
        for q0, q1, a, b in self.qseg.cpu().tolist():
            for k0, k1, t in self.kr[a:b].cpu().tolist():
                out.append((q0, q1, k0, k1, t))
        return out


def spec_from_triples(triples: list[tuple[int, int, int, int, int]], total: int, total_k: int | None = None) -> AttnSpec:
    """Build both groupings from ``(q0, q1, k0, k1, type)`` triples (``total_k`` defaults to
    ``total``; it differs when the keys are gathered from other context-parallel ranks)."""
    by_q: dict[tuple[int, int], list[tuple[int, int, int]]] = {}
    by_k: dict[tuple[int, int], list[tuple[int, int, int]]] = {}
    for q0, q1, k0, k1, t in triples:
        if q1 <= q0 or k1 <= k0:
            continue
        by_q.setdefault((q0, q1), []).append((k0, k1, t))
        by_k.setdefault((k0, k1), []).append((q0, q1, t))

    def group(d: dict) -> tuple[np.ndarray, np.ndarray]:
        seg, items = [], []
        for (a, b), lst in d.items():
            seg.append((a, b, len(items), len(items) + len(lst)))
            items.extend(lst)
        return np.asarray(seg, dtype=np.int32).reshape(-1, 4), np.asarray(items, dtype=np.int32).reshape(-1, 3)

    qseg, kr = group(by_q)
    kseg, qr = group(by_k)
    mq = int((qseg[:, 1] - qseg[:, 0]).max()) if len(qseg) else 0
    mk = int((kseg[:, 1] - kseg[:, 0]).max()) if len(kseg) else 0
    return AttnSpec(torch.from_numpy(qseg), torch.from_numpy(kr), torch.from_numpy(kseg), torch.from_numpy(qr), total,
                    total if total_k is None else total_k, mq, mk, _tiles(qseg, FWD_Q_TILE, kr, True),
                    _tiles(kseg, BWD_K_TILE, qr, False), _tiles(kseg, BWD_K_TILE_TC, qr, False))


FWD_Q_TILE = 128
BWD_K_TILE = 64
BWD_K_TILE_TC = 128


def _tiles(seg: np.ndarray, bs: int, items: np.ndarray | None = None, fwd: bool = True) -> torch.Tensor:
    """(segment, tile start) work list, heaviest tiles first: under causal masks the tiles at the
    end of a long sequence see the most keys (forward) / the first key tiles are seen by the most
    queries (backward), and starting them first keeps the last wave of CTAs short."""
    rows, work = [], []
    its = items.tolist() if items is not None else []
    for i, (s0, s1, r0, r1) in enumerate(seg.tolist()):
        for a in range(s0, s1, bs):
            w = 0
            for x0, x1, t in its[r0:r1]:
                if fwd:  # keys seen by q rows [a, a + bs) of segment (s0, s1)
                    e = min(a + bs, s1)
                    w += max(0, min(x1, x0 + (e - s0)) - x0) if t == 1 else x1 - x0
                else:  # q rows that see key tile [a, a + bs) of segment (s0, s1)
                    w += max(0, x1 - (x0 + max(0, a - s0))) if t == 1 else x1 - x0
            rows.append((i, a))
            work.append(w)
    order = sorted(range(len(rows)), key=lambda j: -work[j])
    return torch.tensor([rows[j] for j in order], dtype=torch.int32).reshape(-1, 2)


def causal_spec_from_cu_seqlens(cu_seqlens: list[int] | np.ndarray) -> AttnSpec:
    cu = [int(x) for x in cu_seqlens]
    return spec_from_triples([(a, b, a, b, 1) for a, b in zip(cu[:-1], cu[1:])], cu[-1])


def tree_spec(q_ranges, k_ranges, types, total: int) -> AttnSpec:  # noqa: ANN001
    return spec_from_triples([(q[0], q[1], k[0], k[1], int(t)) for q, k, t in zip(q_ranges, k_ranges, types)], total)


def dense_mask(spec: AttnSpec) -> torch.Tensor:
    """(T, T) boolean visibility mask (oracle use only)."""
    m = torch.zeros(spec.total_q, spec.total_k, dtype=torch.bool)
    for q0, q1, k0, k1, t in spec.triples():
        if t == 0:
            m[q0:q1, k0:k1] = True
        else:
            i = torch.arange(q1 - q0)[:, None]
            j = torch.arange(k1 - k0)[None, :]
            m[q0:q1, k0:k1] |= j <= i
    return m

"""Context parallelism: each rank of a CP group holds a zigzag slice of every sequence.

Reference: ``cp_size`` (``axrl/configs.py:382``), the zigzag two-chunk split of
``axrl/utils/megatron/pack_utils.py:35-36,91-106`` and the CP output all-gather of
``pack_utils.py:156-161``; Magi attention handles CP for prefix trees
(``axrl/utils/megatron/magi_forward.py:445-466``).

Split.  Each packed row is padded to a multiple of ``2*cp`` and cut into ``2*cp`` equal chunks;
rank ``r`` keeps chunks ``r`` and ``2*cp-1-r`` (early and late tokens, so causal work is balanced).
Every rank's local stream is the concatenation, row by row, of its two chunks, so all ranks have
the same stream length ``L``.

Attention.  Queries stay local; keys and values are all-gathered over the CP group into a
``cp*L`` stream (rank-major), and the range list is rewritten in those coordinates: a row's range
triples (flat causal, or a prefix tree's full-to-ancestors + causal-self ranges) are cut at chunk
boundaries; a causal self range becomes ``full`` for earlier chunks and ``causal`` on the
diagonal chunk.  The gather's backward reduce-scatters the key/value gradients to their owners.

Loss.  A rank trains on its own tokens (its loss mask is restricted to them); gradients are then
summed over the CP group, and per-token log-probs are assembled by summing the ranks' disjoint
parts.  Token-level loss aggregation is exact under this split; sequence-level ratios (GSPO) would
need cross-rank sums and are rejected.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from axrl_b200.configs import IGNORE_INDEX
from axrl_b200.ops.attention_spec import spec_from_triples


@dataclass
class CPContext:
    size: int = 1
    rank: int = 0
    group: Any = None
    comm: Any = None

    @property
    def enabled(self) -> bool:
        return self.size > 1

    @classmethod
    def from_group(cls, group: Any) -> "CPContext":
        if group is None or dist.get_world_size(group) == 1:
            return cls()
        from axrl_b200.parallel.tensor_parallel import TorchTPComm

        comm = TorchTPComm(group)
        return cls(size=comm.size, rank=comm.rank, group=group, comm=comm)


class _GatherKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):  # noqa: ANN001, ANN205
        ctx.comm = comm
        T = x.shape[0]
        return comm.all_gather_rows(x.reshape(T, -1)).view(T * comm.size, *x.shape[1:])

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        n = g.shape[0] // ctx.comm.size
        return ctx.comm.reduce_scatter_rows(g.reshape(g.shape[0], -1).contiguous()).view(n, *g.shape[1:]), None


def gather_kv(x: torch.Tensor, cp: CPContext) -> torch.Tensor:
    """(L, H, D) local keys or values -> (cp*L, H, D) in rank-major order."""
    return _GatherKV.apply(x.contiguous(), cp.comm) if cp.enabled else x


@dataclass
class CPSeqLayout:
    """Where every token of the rank-major ``cp*L`` stream sits in its sequence.

    ``perm[i]`` is the stream index of the i-th token in sequence order (rows one after the other,
    each row's 2*cp chunks in order, padding at the row's end); ``segs`` are the rows' (start, end)
    in that order.  Sequence mixers that need whole sequences (Gated DeltaNet) use it."""

    perm: torch.Tensor  # (cp*L,) int64
    segs: list[tuple[int, int]]


def _a2a(x: torch.Tensor, group: Any) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=group)
    return out


class _SeqToHeads(torch.autograd.Function):
    """(L, P, C) local rows x head groups -> (P*L, C): head group ``rank`` of every rank's rows,
    rank-major (an all-to-all; Ulysses-style exchange of sequence shards for head shards)."""

    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        L, P, C = x.shape
        return _a2a(x.transpose(0, 1), group).reshape(P * L, C)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        PL, C = g.shape
        P = dist.get_world_size(ctx.group)
        return _a2a(g.reshape(P, PL // P, C), ctx.group).transpose(0, 1), None


class _HeadsToSeq(torch.autograd.Function):
    """Inverse of :class:`_SeqToHeads`: (P*L, C) rows of this rank's head group -> (L, P, C)."""

    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        PL, C = x.shape
        P = dist.get_world_size(group)
        return _a2a(x.reshape(P, PL // P, C), group).transpose(0, 1)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        L, P, C = g.shape
        return _a2a(g.transpose(0, 1), ctx.group).reshape(P * L, C), None


def seq_to_heads(x: torch.Tensor, cp: CPContext) -> torch.Tensor:
    return _SeqToHeads.apply(x, cp.group)


def heads_to_seq(x: torch.Tensor, cp: CPContext) -> torch.Tensor:
    return _HeadsToSeq.apply(x, cp.group)


def _row_triples(info, n: int) -> list[tuple[int, int, int, int, int]]:  # noqa: ANN001
    if info is None:
        return [(0, n, 0, n, 1)]
    return [(q0, q1, k0, k1, int(t)) for (q0, q1), (k0, k1), t in zip(info.q_ranges, info.k_ranges, info.attn_type_map)]


def pack_rows_cp(batch, rows: list[int], cp: CPContext):  # noqa: ANN001, ANN201
    """This CP rank's zigzag slice of ``rows`` as a PackedMicroBatch whose spec addresses the
    all-gathered keys."""
    from axrl_b200.train.packing import TOKEN_KEYS_F32, PackedMicroBatch, _row_valid

    P, r = cp.size, cp.rank
    nch = 2 * P
    infos = batch.objects.get("merge_info") or [None] * len(batch)
    fields = {k: [] for k in TOKEN_KEYS_F32 if k in batch.tensors}
    ids, pos, lab, lm, trow, tcol = [], [], [], [], [], []
    plan = []  # per row: (row-local triples, chunk size, row base in every rank's stream)
    base = 0
    row_len = []
    for li, rr in enumerate(rows):
        info = infos[rr]
        n = info.total_padded if info is not None else _row_valid(batch, rr)
        npad = -(-n // nch) * nch
        c = npad // nch
        tri = _row_triples(info, n)
        if npad > n:
            tri.append((n, npad, n, npad, 1))  # padding tokens attend among themselves
        for k in (r, nch - 1 - r):
            a, b = k * c, (k + 1) * c
            va, vb = min(a, n), min(b, n)
            ids.append(batch["input_ids"][rr, va:vb].long())
            pos.append(batch["position_ids"][rr, va:vb].long())
            lab.append(batch["labels"][rr, va:vb].long())
            lm.append(batch["loss_mask"][rr, va:vb].bool())
            for f in fields:
                fields[f].append(batch[f][rr, va:vb].float())
            trow.append(torch.full((vb - va,), li, dtype=torch.int64))
            tcol.append(torch.arange(va, vb))
            pad = b - vb
            if pad:
                ids.append(torch.zeros(pad, dtype=torch.int64))
                pos.append(torch.arange(max(n, a), max(n, a) + pad))
                lab.append(torch.full((pad,), IGNORE_INDEX, dtype=torch.int64))
                lm.append(torch.zeros(pad, dtype=torch.bool))
                for f in fields:
                    fields[f].append(torch.zeros(pad))
                trow.append(torch.full((pad,), -1, dtype=torch.int64))
                tcol.append(torch.zeros(pad, dtype=torch.int64))
        plan.append((tri, c, base))
        row_len.append(n)
        base += 2 * c
    L = base

    def owner(k: int) -> tuple[int, int]:  # chunk -> (rank, 0 first / 1 second chunk of that rank)
        return (k, 0) if k < P else (nch - 1 - k, 1)

    perm = []
    for (_, c, rb) in plan:
        for k in range(nch):
            rk, half = owner(k)
            perm.append(torch.arange(rk * L + rb + half * c, rk * L + rb + (half + 1) * c))
    segs, s0 = [], 0
    for (_, c, _) in plan:
        segs.append((s0, s0 + nch * c))
        s0 += nch * c
    triples = []
    for tri, c, rb in plan:
        def local_q(k: int) -> int | None:  # local stream offset of chunk k (None: not held here)
            rk, half = owner(k)
            return rb + half * c if rk == r else None

        def glob_k(k: int) -> int:
            rk, half = owner(k)
            return rk * L + rb + half * c

        for q0, q1, k0, k1, t in tri:
            if t != 0:
                assert (q0, q1) == (k0, k1), "context parallelism supports causal self ranges only"
            for kq in range(q0 // c, -(-q1 // c)):
                lq = local_q(kq)
                if lq is None:
                    continue
                qa, qb = max(q0, kq * c), min(q1, (kq + 1) * c)
                if qa >= qb:
                    continue
                for kk in range(k0 // c, -(-k1 // c)):
                    ka, kb = max(k0, kk * c), min(k1, (kk + 1) * c)
                    if ka >= kb:
                        continue
                    if t == 0 or kk < kq:
                        typ = 0
                    elif kk == kq:
                        typ = 1
                    else:
                        continue
                    triples.append((lq + qa - kq * c, lq + qb - kq * c, glob_k(kk) + ka - kk * c, glob_k(kk) + kb - kk * c, typ))
    spec = spec_from_triples(triples, L, L * P)
    spec.seq_layout = CPSeqLayout(torch.cat(perm) if perm else torch.zeros(0, dtype=torch.int64), segs)
    return PackedMicroBatch(rows=list(rows), row_len=row_len, row_off=[0] * len(rows), ids=torch.cat(ids), pos=torch.cat(pos).int(),
                            labels=torch.cat(lab), loss_mask=torch.cat(lm), token_row=torch.cat(trow), spec=spec,
                            fields={k: torch.cat(v) for k, v in fields.items()},
                            merge_info=[infos[rr] for rr in rows] if any(infos[rr] is not None for rr in rows) else None,
                            token_col=torch.cat(tcol))


def local_token_mask(mb, width: int) -> torch.Tensor:  # noqa: ANN001
    """(rows, width) bool: the positions whose tokens this CP rank holds."""
    m = torch.zeros((len(mb.rows), width), dtype=torch.bool, device=mb.token_row.device)
    keep = mb.token_row >= 0
    m[mb.token_row[keep], mb.token_col[keep]] = True
    return m

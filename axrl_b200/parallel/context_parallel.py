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

Ring attention (the default when the spec carries per-source tables).  Instead of waiting for the
whole gather, each rank passes its K/V chunk around the ring (send to rank+1, receive from rank-1,
NCCL point-to-point over NVLink on NCCL's stream) and attends to the chunk it holds while the next
one is in flight; the P partial (o, lse) pairs are merged with log-sum-exp weights.  The backward
walks the ring the other way round: at step j a rank computes the dK/dV contribution for the chunk
of rank ``rank-j-1`` (against the final o and lse, which is exact), adds the partial sum received
from rank-1, and forwards it, so the key/value gradients arrive at their owners as a ring
reduce-scatter overlapped with the attention backward; dQ accumulates in fp32 across sources.

Loss.  A rank trains on its own tokens (its loss mask is restricted to them); gradients are then
summed over the CP group, and per-token log-probs are assembled by summing the ranks' disjoint
parts.  Token-level loss aggregation is exact under this split; sequence-level ratios (GSPO) would
need cross-rank sums and are rejected.
"""

from __future__ import annotations

import os
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


class _Ring:
    """Neighbour exchange on the CP ring: every rank sends to ``rank+1`` and receives from
    ``rank-1`` in one batched point-to-point call (NCCL runs it on its own stream; ``wait`` makes
    the current stream wait for it)."""

    def __init__(self, cp: CPContext) -> None:
        P, r = cp.size, cp.rank
        self.group = cp.group
        self.nxt = dist.get_global_rank(cp.group, (r + 1) % P)
        self.prv = dist.get_global_rank(cp.group, (r - 1) % P)

    def shift(self, tensors: tuple[torch.Tensor, ...]) -> "_Pending":
        recv = tuple(torch.empty_like(t) for t in tensors)
        ops = [dist.P2POp(dist.isend, t, self.nxt, self.group, tag=i) for i, t in enumerate(tensors)]
        ops += [dist.P2POp(dist.irecv, t, self.prv, self.group, tag=i) for i, t in enumerate(recv)]
        return _Pending(dist.batch_isend_irecv(ops), tensors, recv)


class _Pending:
    def __init__(self, works: list, sent: tuple, recv: tuple) -> None:
        self.works, self.sent, self.recv = works, sent, recv

    def wait(self) -> tuple[torch.Tensor, ...]:
        for w in self.works:
            w.wait()
        self.sent = None  # the send buffers may be reused from here on
        return self.recv


def _stash_pop(stash, spec, q):  # noqa: ANN001, ANN202
    from axrl_b200.ops.core import AttnStash

    if stash is None or AttnStash.pushing:
        return None
    key = (id(spec), tuple(q.shape))
    lst = stash.items.get(key)
    if not lst:
        return None
    hit = lst.pop(0)
    if not lst:
        del stash.items[key]
    return hit


class _RingAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, spec, cp, scale, stash):  # noqa: ANN001, ANN205
        from axrl_b200.ops import core as ops

        P, r = cp.size, cp.rank
        srcs = spec.cp_sources
        hit = _stash_pop(stash, spec, q)
        ring = _Ring(cp)
        chunks: list = [None] * P
        chunks[r] = (k, v)
        cur, parts = (k, v), []
        for step in range(P):
            s = (r - step) % P
            pend = ring.shift(cur) if step < P - 1 else None
            if hit is None:
                parts.append(ops.attn_partial(q, cur[0], cur[1], srcs[s], scale))
            if pend is not None:
                cur = pend.wait()
                chunks[(r - step - 1) % P] = cur
        if hit is None:
            o, lse2 = ops.attn_merge(parts)
            from axrl_b200.ops.core import AttnStash

            if stash is not None and AttnStash.pushing:
                stash.items.setdefault((id(spec), tuple(q.shape)), []).append((o, lse2))
        else:
            o, lse2 = hit
        ctx.save_for_backward(q, o, lse2, *[c[0] for c in chunks], *[c[1] for c in chunks])
        ctx.spec, ctx.cp, ctx.scale = spec, cp, scale
        return o

    @staticmethod
    def backward(ctx, do):  # noqa: ANN001, ANN205
        from axrl_b200.ops import core as ops

        cp, scale, srcs = ctx.cp, ctx.scale, ctx.spec.cp_sources
        P, r = cp.size, cp.rank
        q, o, lse2, *kv = ctx.saved_tensors
        ks, vs = kv[:P], kv[P:]
        do = do.contiguous()
        dsum = ops.attn_bwd_dsum(o, do)
        dq_acc = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        ring = _Ring(cp)
        pend = None
        for j in range(P):
            c = (r - j - 1) % P  # j = P-1: this rank's own chunk, the last to be completed
            dk, dv = ops.attn_bwd_partial(do, q, ks[c], vs[c], lse2, dsum, dq_acc, srcs[c], scale)
            if pend is not None:
                rk, rv = pend.wait()
                dk, dv = dk + rk, dv + rv
            pend = ring.shift((dk, dv)) if j < P - 1 else None
        return dq_acc.to(q.dtype), dk, dv, None, None, None, None


def ring_attention_supported(spec, cp: CPContext) -> bool:  # noqa: ANN001
    """Ring attention needs the per-source tables and non-deterministic dQ (the deterministic
    backward owns dQ per query tile in one kernel over all keys: the gathered path keeps it);
    ``AXRL_CP_ATTN=gather`` selects the gathered path."""
    if not cp.enabled or getattr(spec, "cp_sources", None) is None or len(spec.cp_sources) != cp.size or cp.size > 16:
        return False
    if os.environ.get("AXRL_CP_ATTN", "ring") == "gather":
        return False
    if spec.qseg.is_cuda or torch.cuda.is_available():
        from axrl_b200.ops import _ext

        try:
            return not _ext.ext().attn_deterministic()
        except Exception:  # noqa: BLE001 - no extension on this host: the CPU path has no such mode
            return True
    return True


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec, cp: CPContext, scale: float | None = None,  # noqa: ANN001
                   stash=None) -> torch.Tensor:  # noqa: ANN001
    """Attention of the local queries over the keys of every CP rank, overlapped with the K/V ring
    exchange.  q: (L, Hq, D) local; k, v: (L, Hkv, D) local; ``spec.cp_sources[s]`` addresses the
    keys of rank s in that rank's stream coordinates."""
    import math

    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if q.is_cuda and not spec.qseg.is_cuda:
        spec = spec.to(q.device)
    return _RingAttn.apply(q.contiguous(), k.contiguous(), v.contiguous(), spec, cp, scale, stash)


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
    by_src: list[list] = [[] for _ in range(P)]
    for q0, q1, k0, k1, t in triples:  # a triple's keys never cross a chunk, so one source each
        s = k0 // L
        by_src[s].append((q0, q1, k0 - s * L, k1 - s * L, t))
    spec.cp_sources = [spec_from_triples(t, L, L) for t in by_src]
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

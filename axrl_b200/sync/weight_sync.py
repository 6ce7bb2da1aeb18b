"""Trainer -> rollout weight sync over NVLink symmetric memory.

Reference: ``SGLangTensorWeightUpdater`` (colocated: bridge export + buckets + CUDA IPC,
``axrl/utils/megatron/sglang_weight_updater.py:60-271``) and ``SGLangDistributedWeightUpdater``
(disaggregated: rank-0 NCCL broadcast, :274-338), timed in
``benchmark/weight_update/run_fp8_weight_sync_benchmark.py``.

Every rank of the sync group allocates one symmetric buffer of the same size: trainer ranks
keep their TP shard of all parameters in it (bf16, flat, :func:`build_layout` order); rollout
ranks receive their shard in it (bf16, or e4m3 + fp32 128x128 block scales).  ``push()`` runs
one kernel per trainer rank that writes every tile it owns straight into the destination
ranks' buffers (P2P stores), then a symmetric-memory barrier publishes the new weights.
The NCCL baseline (:meth:`push_nccl`) gathers full tensors to each destination with
``all_gather`` + a local reshard, for comparison.
"""

from __future__ import annotations

import time

import numpy as np
import torch
import torch.distributed as dist

from axrl_b200.ops import _ext
from axrl_b200.sync.plan import TILE, ParamSpec, build_layout, build_tiles, split_modes


class WeightSyncer:
    def __init__(self, specs: list[ParamSpec], *, src_tp: int, src_ranks: list[int], dst_tp: int, dst_groups: list[list[int]],
                 fp8: bool = False, group=None, device=None) -> None:  # noqa: ANN001
        """``src_ranks[i]`` holds trainer TP shard i; each ``dst_groups[e]`` lists the global ranks of
        rollout engine e (its TP shards in order).  A rank may appear in both roles."""
        import torch.distributed._symmetric_memory as symm_mem

        self.specs, self.src_tp, self.dst_tp, self.fp8 = specs, src_tp, dst_tp, fp8
        self.rank = dist.get_rank()
        self.group = group
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.src_layout = build_layout(specs, src_tp, fp8=False)
        # destination region follows the source region, so a rank can hold both roles
        self.dst_base = -(-self.src_layout.nbytes // 4096) * 4096
        self.dst_layout = build_layout(specs, dst_tp, fp8=fp8, base=self.dst_base)
        nbytes = -(-self.dst_layout.nbytes // 4096) * 4096
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
        gname = (group or dist.group.WORLD).group_name
        self.handle = symm_mem.rendezvous(self.buf, gname)
        self.ptrs = torch.tensor(self.handle.buffer_ptrs, dtype=torch.int64, device=self.device)
        self.src_rank = src_ranks.index(self.rank) if self.rank in src_ranks else None
        self.tiles_copy = self.tiles_q8 = None
        if self.src_rank is not None:
            tiles = [build_tiles(specs, src_tp, dst_tp, self.src_layout, self.dst_layout, self.src_rank, grp, fp8) for grp in dst_groups]
            allt = np.concatenate(tiles, 0) if tiles else np.zeros((0, 10), np.int64)
            c, q = split_modes(allt)
            self.tiles_copy = torch.from_numpy(c).to(self.device)
            self.tiles_q8 = torch.from_numpy(q).to(self.device)
        self.bytes_pushed = 0 if self.src_rank is None else int(self._pushed_bytes())
        # NCCL baseline: every trainer shard is broadcast to all ranks, then each destination rank
        # reshards locally with the same tile kernel (its own tiles only)
        self.src_ranks = list(src_ranks)
        self._nccl_tiles: list[tuple[torch.Tensor, torch.Tensor]] = []
        my_groups = [g for g in dst_groups if self.rank in g]
        for i in range(len(src_ranks)):
            tl = [build_tiles(specs, src_tp, dst_tp, self.src_layout, self.dst_layout, i, g, fp8) for g in my_groups]
            allt = np.concatenate(tl, 0) if tl else np.zeros((0, 10), np.int64)
            allt = allt[allt[:, 2] == self.rank]
            c, q = split_modes(allt)
            self._nccl_tiles.append((torch.from_numpy(c).to(self.device), torch.from_numpy(q).to(self.device)))

    def _pushed_bytes(self) -> int:
        n = 0
        for t in (self.tiles_copy, self.tiles_q8):
            if t is not None and t.numel():
                rows, cols = t[:, 5].cpu(), t[:, 6].cpu()
                n += int((rows * cols).sum()) * (1 if t is self.tiles_q8 else 2)
        return n

    def src_view(self) -> torch.Tensor:
        """bf16 view of the whole buffer (tile offsets are absolute element offsets)."""
        return self.buf.view(torch.bfloat16)

    def param_view(self, name: str, role: str = "src") -> torch.Tensor:
        lay = self.src_layout if role == "src" else self.dst_layout
        r, c = lay.shapes[name]
        if role == "src" or name not in lay.scale_offsets:
            return self.buf.view(torch.bfloat16)[lay.offsets[name]: lay.offsets[name] + r * c].view(r, c)
        return self.buf[lay.offsets[name]: lay.offsets[name] + r * c].view(torch.float8_e4m3fn).view(r, c)

    def scale_view(self, name: str) -> torch.Tensor:
        lay = self.dst_layout
        r, c = lay.shapes[name]
        n = -(-r // TILE) * -(-c // TILE)
        return self.buf[lay.scale_offsets[name]: lay.scale_offsets[name] + 4 * n].view(torch.float32).view(-(-r // TILE), -(-c // TILE))

    def push_nccl(self) -> float:
        """Baseline: NCCL broadcast of every trainer shard + local reshard/quantise on each
        destination; returns device seconds (this rank)."""
        e = _ext.ext()
        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = -(-self.src_layout.nbytes // 16) * 16
        recv = torch.empty(n, dtype=torch.uint8, device=self.device)
        local = torch.full((len(self.handle.buffer_ptrs),), self.buf.data_ptr(), dtype=torch.int64, device=self.device)
        dist.barrier(group=self.group)
        s.record()
        for i, r in enumerate(self.src_ranks):
            shard = self.buf[:n] if self.rank == r else recv
            dist.broadcast(shard, src=r, group=self.group)
            copy_t, q_t = self._nccl_tiles[i]
            src = shard.view(torch.bfloat16)
            if copy_t.numel():
                e.sync_push(copy_t, src, local, 0)
            if q_t.numel():
                e.sync_push(q_t, src, local, 1)
        t.record()
        t.synchronize()
        dist.barrier(group=self.group)
        return s.elapsed_time(t) / 1000.0

    def push(self) -> float:
        """One full reshard + (quantise) + push; returns device seconds (this rank)."""
        e = _ext.ext()
        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.handle.barrier(channel=0)  # destinations finished reading the previous weights
        s.record()
        if self.src_rank is not None:
            src = self.src_view()
            if self.tiles_copy.numel():
                e.sync_push(self.tiles_copy, src, self.ptrs, 0)
            if self.tiles_q8.numel():
                e.sync_push(self.tiles_q8, src, self.ptrs, 1)
        t.record()
        self.handle.barrier(channel=1)  # every tile has landed
        t.synchronize()
        return s.elapsed_time(t) / 1000.0

"""Tensor-parallel rollout: collectives for a decode/prefill step sharded over TP ranks.

Reference: SGLang engines with ``tp_size`` (``RolloutWorkerConfig``, ``axrl/configs.py:210-214``) and
their custom all-reduce fused with RMSNorm.  Each TP rank runs its own :class:`RolloutEngine` over a
TP-sharded model (local heads / FFN columns, local KV heads) with the same requests and seeds; the
rank-local scheduler decisions therefore agree.  Per layer:

* QKV / gate-up GEMMs on the local shards (no communication);
* O / down projections write their partial sums into a symmetric buffer, and ONE kernel
  (``csrc/kernels/rollout_tp.cu``) all-reduces them over NVLink (P2P loads), adds the residual
  and applies the next RMSNorm;
* the LM head runs on the local vocabulary shard; the logits rows are all-gathered so every rank
  samples the same token (identical RNG streams).

The embedding table is kept whole on every rank (a lookup needs no communication), which also
makes the number of all-reduces per forward even, so alternating the two partial buffers keeps a
GEMM from overwriting a partial that a peer may still be reading.  All kernels are graph-safe
(device-side epochs) and their waits are bounded; :meth:`RolloutTP.check` raises on a timeout.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from axrl_b200.ops import _ext

_BLOCKS, _MAXTP = 32, 8


class RolloutTP:
    def __init__(self, group: Any, hidden: int, vocab_shard: int, max_rows: int, max_batch: int, dtype: torch.dtype = torch.bfloat16) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.size <= _MAXTP
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device, self.H, self.Vs = dev, hidden, vocab_shard
        self.max_rows, self.max_batch = max_rows, max_batch
        gname = (group or dist.group.WORLD).group_name
        self.part = symm_mem.empty(2 * max_rows * hidden, dtype=dtype, device=dev)
        self.logit = symm_mem.empty(2 * max_batch * vocab_shard, dtype=dtype, device=dev)
        self.flags = symm_mem.empty(_BLOCKS * _MAXTP, dtype=torch.int32, device=dev)
        self.flags.zero_()
        hp, hl, hf = (symm_mem.rendezvous(t, gname) for t in (self.part, self.logit, self.flags))
        self.part_ptrs = torch.tensor(hp.buffer_ptrs, dtype=torch.int64)
        self.logit_ptrs = torch.tensor(hl.buffer_ptrs, dtype=torch.int64)
        self.flag_ptrs = torch.tensor(hf.buffer_ptrs, dtype=torch.int64)
        self.ctr = torch.zeros(_BLOCKS, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.timeout_ns = int(float(os.environ.get("AXRL_ROLLOUT_TP_TIMEOUT_S", "30")) * 1e9)
        self.parity = 0
        hf.barrier(channel=0)

    def check(self) -> None:
        if int(self.status.item()):
            raise RuntimeError("rollout TP collective timed out (a peer engine is missing or late)")

    def partial_buffer(self, rows: int) -> torch.Tensor:
        """Where the next row-parallel GEMM writes its (rows, H) partial (alternating halves)."""
        assert rows <= self.max_rows, f"{rows} rows exceed the TP buffer ({self.max_rows})"
        off = self.parity * self.max_rows * self.H
        return self.part[off:off + rows * self.H].view(rows, self.H)

    def allreduce_rms(self, rows: int, residual: torch.Tensor | None, norm_w: torch.Tensor, eps: float,
                      want_h: bool = True) -> tuple[torch.Tensor | None, torch.Tensor]:
        """h = residual + sum of every rank's partial; x = RMSNorm(h) * norm_w.  Returns (h, x)."""
        off = self.parity * self.max_rows * self.H
        self.parity ^= 1
        out_h = torch.empty(rows, self.H, dtype=self.part.dtype, device=self.device) if want_h else None
        out_x = torch.empty(rows, self.H, dtype=self.part.dtype, device=self.device)
        _ext.ext().tp_ar_rms(self.part_ptrs, off, rows, self.H, residual, norm_w, eps, out_h, out_x, self.flag_ptrs, self.flags, self.ctr,
                             self.rank, self.timeout_ns, self.status)
        return out_h, out_x

    def logits_buffer(self, rows: int) -> torch.Tensor:
        assert rows <= self.max_batch
        return self.logit[:rows * self.Vs].view(rows, self.Vs)

    def gather_logits(self, rows: int) -> torch.Tensor:
        out = torch.empty(rows, self.Vs * self.size, dtype=self.logit.dtype, device=self.device)
        _ext.ext().tp_gather_cols(self.logit_ptrs, 0, rows, self.Vs, out, self.flag_ptrs, self.flags, self.ctr, self.rank, self.timeout_ns,
                                  self.status)
        return out

"""NVLink tensor-parallel collectives with the GEMM split into per-rank row chunks that overlap
the transfers (all-gather -> GEMM and GEMM -> reduce-scatter over peer memory).

Reference counterpart: Megatron's sequence-parallel Column/RowParallelLinear, which calls NCCL
all-gather / reduce-scatter around cuBLAS GEMMs (``axrl/worker/megatron_worker.py:825``).  Here
(``csrc/kernels/tp_comm.cu``):

* all-gather -> GEMM (``ag_linear``): every rank pushes its T/tp input rows into every peer's
  symmetric gather buffer with P2P stores (a comm-stream kernel), while the compute stream runs
  the GEMM on the local rows; each peer's row chunk is multiplied as soon as its arrival flag is
  seen.  The GEMMs read only local memory.
* GEMM -> reduce-scatter (``linear_rs``): the GEMM runs chunk by chunk, peers' chunks first; each
  finished chunk is pushed into its owner's slot while the next chunk computes; the owner sums
  its slots (plus the residual, fused) once every peer's slot has arrived.
* backward passes use the same two patterns in the other direction (dgrad -> reduce-scatter with
  the input re-gathered for the weight gradient under the dgrad GEMMs; all-gather of dy -> dgrad).
* fused GEMM -> reduce-scatter (``AXRL_TP_FUSED=1``): ONE kernel (``csrc/kernels/tcgemm.cu``, mode
  SLOTS) computes every output tile on the tensor cores and stores it straight into its owner's
  receive slot over NVLink, so the transfer of each tile overlaps the MMAs of the next; the kernel
  itself performs the free / data handshakes of the channel, and the owner then sums its slots
  (plus the residual).
* fused all-gather -> GEMM (default; ``AXRL_TP_FUSED_AG=0`` disables): ONE kernel (mode AGATHER) whose copy warps pull
  the other ranks' rows from their gather buffers over NVLink into this rank's (each row crosses the
  link once) while its MMAs start on the local rows; the TMA producer waits per source chunk for the
  copies to complete.

All waits are bounded; :meth:`P2PTPComm.check` raises if a peer timed out.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from axrl_b200.ops import _ext
from axrl_b200.parallel.tensor_parallel import TorchTPComm, TPComm

CH_AG, CH_RS, CH_AGF = 0, 1, 2
_K_CHANNELS, _K_MAXTP = 32, 8


class P2PTPComm(TPComm):
    def __init__(self, group: Any, cap_tokens: int | None = None, hidden: int | None = None, push_ctas: int = 32) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.size <= _K_MAXTP
        self.fallback = TorchTPComm(group)
        self.cap_tokens = cap_tokens or int(os.environ.get("AXRL_TP_CAP_TOKENS", 16384 + 1024))
        self.hidden = hidden or int(os.environ.get("AXRL_TP_HIDDEN", 4096))
        self.timeout_ns = int(float(os.environ.get("AXRL_TP_TIMEOUT_S", "60")) * 1e9)
        self.push_ctas = push_ctas
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        cap = self.cap_tokens * self.hidden
        gname = (group or dist.group.WORLD).group_name
        self.ag = symm_mem.empty(cap, dtype=torch.bfloat16, device=dev)
        self.rs = symm_mem.empty(cap, dtype=torch.bfloat16, device=dev)
        self.flags = symm_mem.empty(_K_CHANNELS * _K_MAXTP, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.h_ag = symm_mem.rendezvous(self.ag, gname)
        self.h_rs = symm_mem.rendezvous(self.rs, gname)
        self.h_flags = symm_mem.rendezvous(self.flags, gname)
        self.ag_ptrs = torch.tensor(self.h_ag.buffer_ptrs, dtype=torch.int64)
        self.rs_ptrs = torch.tensor(self.h_rs.buffer_ptrs, dtype=torch.int64)
        self.flag_ptrs = torch.tensor(self.h_flags.buffer_ptrs, dtype=torch.int64)
        self.rs_ptrs_dev = self.rs_ptrs.to(dev)
        self.flag_ptrs_dev = self.flag_ptrs.to(dev)
        # one-kernel GEMM -> reduce-scatter: opt-in (slower than the chunked path at 2 GPUs);
        # one-kernel all-gather -> GEMM: default (the fastest of the three at 2 GPUs)
        self.fused = os.environ.get("AXRL_TP_FUSED", "0") == "1"
        self.fused_ag = self.fused or os.environ.get("AXRL_TP_FUSED_AG", "1") == "1"
        if self.fused_ag:  # all-gather -> GEMM in one kernel: a gather buffer the kernels pull from
            self.agf = symm_mem.empty(cap, dtype=torch.bfloat16, device=dev)
            self.h_agf = symm_mem.rendezvous(self.agf, gname)
            self.agf_ptrs_dev = torch.tensor(self.h_agf.buffer_ptrs, dtype=torch.int64).to(dev)
            self.ag_cnt = torch.zeros(_K_MAXTP, dtype=torch.int32, device=dev)
            self.ag_calls = 0
            self.ag_last_epoch = 0
        self.stage = torch.empty(2, cap // self.size, dtype=torch.bfloat16, device=dev)
        self.ticket = torch.zeros(_K_CHANNELS, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        self.comm_stream = torch.cuda.Stream(device=dev)
        self.h_flags.barrier(channel=0)  # every rank's flags are zero before any push

    # -------------------------------------------------------------- primitives
    def _next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def _push(self, src: torch.Tensor, chunk_bytes: int, src_stride_bytes: int, dst_ptrs: torch.Tensor, dst_off_bytes: int,
              ch: int, epoch: int, mask: int) -> None:
        _ext.ext().tp_push(src, chunk_bytes, src_stride_bytes, dst_ptrs, dst_off_bytes, self.flag_ptrs, self.flags, ch, epoch,
                           self.rank, mask, self.ticket, self.timeout_ns, self.status, self.push_ctas)

    def _wait(self, ch: int, mask: int, epoch: int) -> None:
        _ext.ext().tp_wait(self.flags, ch, mask & ~(1 << self.rank), epoch, self.timeout_ns, self.status)

    def _fits(self, x: torch.Tensor, rows_total: int) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous() and x.shape[1] % 8 == 0
                and rows_total * x.shape[1] <= self.ag.numel())

    def check(self) -> None:
        """Raise if any bounded wait of this communicator expired (a peer is missing or late)."""
        s = int(self.status.item())
        if s:
            raise RuntimeError(f"TP P2P collective timed out (status {s}: {'free barrier' if s == 1 else 'data arrival'})")

    # -------------------------------------------------------------- plain collectives
    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0]
        if not self._fits(x, n * self.size):
            return self.fallback.all_gather_rows(x)
        C = x.shape[1]
        e = self._next_epoch()
        all_mask = (1 << self.size) - 1
        self._push(x, n * C * 2, 0, self.ag_ptrs, self.rank * n * C * 2, CH_AG, e, all_mask)
        self._wait(CH_AG, all_mask, e)
        return self.ag[:n * self.size * C].view(n * self.size, C).clone()

    def reduce_scatter_rows(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        T = x.shape[0]
        if not self._fits(x, T) or T % self.size:
            out = self.fallback.reduce_scatter_rows(x)
            return out if residual is None else out + residual
        n, C = T // self.size, x.shape[1]
        e = self._next_epoch()
        all_mask = (1 << self.size) - 1
        self._push(x, n * C * 2, n * C * 2, self.rs_ptrs, self.rank * n * C * 2, CH_RS, e, all_mask)
        self._wait(CH_RS, all_mask, e)
        out = torch.empty(n, C, dtype=x.dtype, device=x.device)
        _ext.ext().tp_reduce_slots(self.rs, self.size, n * C, residual, out)
        return out

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.fallback.all_reduce(x)

    # -------------------------------------------------------------- overlapped GEMM pipelines
    def _gather_chunks(self, x_local: torch.Tensor, consume) -> int:  # noqa: ANN001
        """Push ``x_local`` to every rank's gather buffer; call ``consume(src, rows)`` for the local
        chunk immediately and for each peer chunk once it has arrived.  Returns the epoch."""
        n, C = x_local.shape
        e = self._next_epoch()
        cur = torch.cuda.current_stream()
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            self._push(x_local, n * C * 2, 0, self.ag_ptrs, self.rank * n * C * 2, CH_AG, e, (1 << self.size) - 1)
        consume(self.rank, x_local)
        for k in range(1, self.size):
            src = (self.rank - k) % self.size  # rank s pushes to s+1 first
            self._wait(CH_AG, 1 << src, e)
            consume(src, self.ag[src * n * C:(src + 1) * n * C].view(n, C))
        return e

    def _gathered(self, n: int, C: int) -> torch.Tensor:
        return self.ag[:n * self.size * C].view(n * self.size, C)

    def _scatter_chunks(self, n: int, C: int, produce, residual: torch.Tensor | None) -> torch.Tensor:  # noqa: ANN001
        """``produce(owner, out)`` writes the (n, C) partial for ``owner``'s rows into ``out``;
        peers' chunks are produced first and pushed while the next chunk computes."""
        e = self._next_epoch()
        cur = torch.cuda.current_stream()
        events = [None, None]
        nbytes = n * C * 2
        for s in range(self.size):
            owner = (self.rank + 1 + s) % self.size
            if owner == self.rank:
                produce(owner, self.rs[self.rank * n * C:(self.rank + 1) * n * C].view(n, C))
                continue
            buf = self.stage[s % 2, :n * C].view(n, C)
            if events[s % 2] is not None:
                cur.wait_event(events[s % 2])
            produce(owner, buf)
            self.comm_stream.wait_stream(cur)
            with torch.cuda.stream(self.comm_stream):
                self._push(buf, nbytes, 0, self.rs_ptrs, self.rank * nbytes, CH_RS, e, 1 << owner)
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            events[s % 2] = ev
        self._wait(CH_RS, (1 << self.size) - 1, e)
        out = torch.empty(n, C, dtype=torch.bfloat16, device=self.device)
        _ext.ext().tp_reduce_slots(self.rs, self.size, n * C, residual, out)
        cur.wait_stream(self.comm_stream)
        return out

    def fused_rs_ok(self, x: torch.Tensor, w: torch.Tensor) -> bool:
        """Shapes the fused tcgen05 GEMM -> reduce-scatter kernel accepts."""
        T, K = x.shape
        N = w.shape[0]
        return self.fused and T % self.size == 0 and K % 64 == 0 and N % 32 == 0 and T * N <= self.rs.numel()

    def gemm_rs_fused(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        """out (T/tp, N) = RS(x @ w^T) (+ residual), the GEMM tiles stored into the owners' slots."""
        T, N = x.shape[0], w.shape[0]
        n = T // self.size
        e = self._next_epoch()
        _ext.ext().tc_linear_to_slots(x, w, self.rs_ptrs_dev, self.rank, n, self.flag_ptrs_dev, self.flags, CH_RS, e, self.ticket,
                                      self.timeout_ns, self.status)
        self._wait(CH_RS, (1 << self.size) - 1, e)
        out = torch.empty(n, N, dtype=torch.bfloat16, device=self.device)
        _ext.ext().tp_reduce_slots(self.rs, self.size, n * N, residual, out)
        return out

    def fused_ag_ok(self, x_local: torch.Tensor, w: torch.Tensor) -> bool:
        """Shapes the one-kernel all-gather -> GEMM accepts."""
        n, K = x_local.shape
        return (self.fused_ag and n % 128 == 0 and K % 8 == 0 and w.shape[0] % 32 == 0 and n * self.size * K <= self.agf.numel()
                and x_local.dtype == torch.bfloat16)

    def ag_gemm_fused(self, x_local: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """y (T, N) = AG(x_local) @ w^T in one kernel: this rank's rows go into its gather buffer, the
        kernel pulls the other ranks' rows over NVLink while it multiplies the local ones."""
        n, K = x_local.shape
        T = n * self.size
        peers = ((1 << self.size) - 1) & ~(1 << self.rank)
        if self.ag_last_epoch:  # every peer has pulled this rank's rows of the previous call
            _ext.ext().tp_wait(self.flags, CH_AGF + 16, peers, self.ag_last_epoch, self.timeout_ns, self.status)
        buf = self.agf[:T * K].view(T, K)
        buf[self.rank * n:(self.rank + 1) * n].copy_(x_local)
        e = self._next_epoch()
        self.ag_calls += 1
        y = torch.empty(T, w.shape[0], dtype=x_local.dtype, device=x_local.device)
        _ext.ext().tc_linear_ag(self.agf, w, y, self.agf_ptrs_dev, self.rank, n, self.flag_ptrs_dev, self.flags, CH_AGF, e, self.ag_cnt,
                                self.ag_calls, self.timeout_ns, self.status)
        self.ag_last_epoch = e
        return y

    def ag_linear(self, x_local: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        T = x_local.shape[0] * self.size
        if not self._fits(x_local.reshape(x_local.shape[0], -1), T) or not w.is_cuda:
            return None  # caller falls back
        return _AGLinear.apply(x_local.contiguous(), w, self)

    def linear_rs(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        T, N = x.shape[0], w.shape[0]
        if T % self.size or T * N > self.rs.numel() or N % 8 or x.dtype != torch.bfloat16 or not w.is_cuda:
            return None  # caller falls back
        return _LinearRS.apply(x.contiguous(), w, residual, self)


def _wgrad(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor):  # noqa: ANN202
    e = _ext.ext()
    main = getattr(w, "main_grad", None)
    if main is not None:
        e.linear_wgrad_acc(dy, x, main)
        return None
    return e.linear_wgrad(dy, x)


class _AGLinear(torch.autograd.Function):
    """y (T, N_l) = AG(x_local) @ w_l^T."""

    @staticmethod
    def forward(ctx, x_local, w, comm):  # noqa: ANN001, ANN205
        n = x_local.shape[0]
        if comm.fused_ag_ok(x_local, w):  # one kernel: peer rows pulled over NVLink under the local MMAs
            y = comm.ag_gemm_fused(x_local, w)
        else:
            y = torch.empty(n * comm.size, w.shape[0], dtype=x_local.dtype, device=x_local.device)
            e = _ext.ext()
            comm._gather_chunks(x_local, lambda src, rows: e.linear_fwd_into(rows, w, y[src * n:(src + 1) * n]))
            torch.cuda.current_stream().wait_stream(comm.comm_stream)
        ctx.save_for_backward(x_local, w)
        ctx.comm = comm
        return y

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x_local, w = ctx.saved_tensors
        comm = ctx.comm
        dy = dy.contiguous()
        n, K = x_local.shape
        e = _ext.ext()
        # re-gather x for the weight gradient (pushed under the dgrad GEMMs)
        ep = comm._next_epoch()
        cur = torch.cuda.current_stream()
        comm.comm_stream.wait_stream(cur)
        with torch.cuda.stream(comm.comm_stream):
            comm._push(x_local, n * K * 2, 0, comm.ag_ptrs, comm.rank * n * K * 2, CH_AG, ep, (1 << comm.size) - 1)
        dx = comm._scatter_chunks(n, K, lambda o, out: e.linear_dgrad_into(dy[o * n:(o + 1) * n], w, out), None)
        comm._wait(CH_AG, (1 << comm.size) - 1, ep)
        dw = _wgrad(dy, comm._gathered(n, K), w) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _LinearRS(torch.autograd.Function):
    """out (n, N) = RS(x @ w_l^T) (+ residual)."""

    @staticmethod
    def forward(ctx, x, w, residual, comm):  # noqa: ANN001, ANN205
        T = x.shape[0]
        n = T // comm.size
        e = _ext.ext()
        if comm.fused_rs_ok(x, w):  # one kernel: tcgen05 tiles stored into the owners' slots over NVLink
            out = comm.gemm_rs_fused(x, w, residual)
        else:
            out = comm._scatter_chunks(n, w.shape[0], lambda o, buf: e.linear_fwd_into(x[o * n:(o + 1) * n], w, buf), residual)
        ctx.save_for_backward(x, w)
        ctx.comm = comm
        ctx.has_res = residual is not None
        return out

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        x, w = ctx.saved_tensors
        comm = ctx.comm
        g = g.contiguous()
        n, N = g.shape
        e = _ext.ext()
        dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        comm._gather_chunks(g, lambda src, rows: e.linear_dgrad_into(rows, w, dx[src * n:(src + 1) * n]))
        torch.cuda.current_stream().wait_stream(comm.comm_stream)
        dw = _wgrad(comm._gathered(n, N), x, w) if ctx.needs_input_grad[1] else None
        return dx, dw, (g if ctx.has_res else None), None

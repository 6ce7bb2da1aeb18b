"""Device-side expert-parallel dispatch/combine over NVLink (``csrc/kernels/ep_comm.cu``).

Per MoE layer, with no host synchronisation:

1. each rank pushes its per-expert row counts into every rank's symmetric count table;
2. ``ep_plan`` derives the receive layout (rows grouped by local expert, then source rank: the
   grouped-GEMM order) and where each of this rank's rows goes;
3. dispatch: P2P stores of every sorted token row into its owner's receive buffer;
4. the grouped expert FFN runs on the receive buffer with the plan's device offsets;
5. combine: P2P stores of every expert output row back into its source's buffer, in the source's
   sorted order; the source applies the routing weights and sums the top-k rows per token.

Backward mirrors it (combine^T = dispatch of the output gradients, dispatch^T = combine of the
input gradients).  Receive buffers have a fixed capacity (``cap_factor`` x the average rows per
rank); a layer whose received rows would exceed it raises before any row moves.

Reference counterpart: Megatron's NCCL all-to-all token dispatcher
(``axrl/worker/megatron_worker.py:833``); :class:`axrl_b200.parallel.expert.TorchEPComm` is that
baseline here.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from axrl_b200.ops import _ext

CH_CNT, CH_A_RECV, CH_A_BACK, CH_B_RECV, CH_B_BACK = 2, 3, 4, 5, 6
_K_CHANNELS, _K_MAX = 32, 8


class _Plan:
    def __init__(self, C: torch.Tensor, E_l: int, n_send: int) -> None:
        P = C.shape[0]
        dev = C.device
        self.C = C
        self.offsets = torch.empty(E_l + 1, dtype=torch.int32, device=dev)
        self.dst_start = torch.empty(C.shape[1], dtype=torch.int32, device=dev)
        self.blk_pos = torch.empty(E_l * P, dtype=torch.int32, device=dev)
        self.blk_src = torch.empty(E_l * P, dtype=torch.int32, device=dev)
        self.totals = torch.empty(2, dtype=torch.int32, device=dev)
        self.n_send = n_send


class P2PEPComm:
    def __init__(self, group: Any, hidden: int | None = None, num_experts: int | None = None, max_rows: int | None = None,
                 cap_factor: float | None = None, ctas: int = 64) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.size <= _K_MAX
        self.hidden = hidden or int(os.environ.get("AXRL_EP_HIDDEN", 2048))
        self.E = num_experts or int(os.environ.get("AXRL_EP_EXPERTS", 128))
        assert self.E % self.size == 0 and self.E % 4 == 0
        self.max_rows = max_rows or int(os.environ.get("AXRL_EP_MAX_ROWS", (16384 + 1024) * 8))  # tokens x top-k per rank
        cf = cap_factor or float(os.environ.get("AXRL_EP_CAP_FACTOR", "2.0"))
        self.cap_recv = int(self.max_rows * cf)
        self.timeout_ns = int(float(os.environ.get("AXRL_EP_TIMEOUT_S", "60")) * 1e9)
        self.ctas = ctas
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        gname = (group or dist.group.WORLD).group_name
        H = self.hidden

        def symm(n, dtype):  # noqa: ANN001, ANN202
            t = symm_mem.empty(n, dtype=dtype, device=dev)
            h = symm_mem.rendezvous(t, gname)
            return t, h, torch.tensor(h.buffer_ptrs, dtype=torch.int64)

        self.cnt, self.h_cnt, self.cnt_ptrs = symm(self.size * self.E, torch.int32)
        self.recv_a, _, self.recv_a_ptrs = symm(self.cap_recv * H, torch.bfloat16)
        self.recv_b, _, self.recv_b_ptrs = symm(self.cap_recv * H, torch.bfloat16)
        self.back_a, _, self.back_a_ptrs = symm(self.max_rows * H, torch.bfloat16)
        self.back_b, _, self.back_b_ptrs = symm(self.max_rows * H, torch.bfloat16)
        self.flags, self.h_flags, self.flag_ptrs = symm(_K_CHANNELS * _K_MAX, torch.int32)
        self.flags.zero_()
        self.ticket = torch.zeros(_K_CHANNELS, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        self.h_flags.barrier(channel=0)

    def _next(self) -> int:
        self.epoch += 1
        return self.epoch

    def _all(self) -> int:
        return ((1 << self.size) - 1) & ~(1 << self.rank)

    def check(self) -> None:
        s = int(self.status.item())
        if s:
            what = {1: "a peer did not free its buffer in time", 2: "data did not arrive in time", 3: "receive capacity exceeded"}
            raise RuntimeError(f"EP P2P transfer failed (status {s}: {what.get(s, '?')})")

    # -------------------------------------------------------------- steps
    def plan(self, exp_sorted: torch.Tensor) -> _Plan:
        e = _ext.ext()
        counts = torch.zeros(self.E, dtype=torch.int32, device=exp_sorted.device)  # no host sync (unlike bincount)
        counts.scatter_add_(0, exp_sorted.long(), torch.ones_like(exp_sorted, dtype=torch.int32))
        ep = self._next()
        e.tp_push(counts, self.E * 4, 0, self.cnt_ptrs, self.rank * self.E * 4, self.flag_ptrs, self.flags, CH_CNT, ep, self.rank,
                  (1 << self.size) - 1, self.ticket, self.timeout_ns, self.status, 1)
        e.tp_wait(self.flags, CH_CNT, self._all(), ep, self.timeout_ns, self.status)
        C = self.cnt.view(self.size, self.E).clone()
        n_send = int(exp_sorted.numel())
        assert n_send <= self.max_rows, "more (token, expert) rows than the EP send buffers hold"
        p = _Plan(C, self.E // self.size, n_send)
        e.ep_plan(C, self.rank, p.offsets, p.dst_start, p.blk_pos, p.blk_src, p.totals)
        # rows this rank receives: one host read per layer, so the expert FFN and the copies out of
        # the receive buffer cover the received rows only, not the whole capacity
        p.n_recv = int(p.totals[0].item())
        if p.n_recv > self.cap_recv:  # the expert FFN would read past the receive buffer
            raise RuntimeError(f"EP receive capacity exceeded: {p.n_recv} rows for {self.cap_recv} (raise AXRL_EP_CAP_FACTOR)")
        return p

    def _transfer(self, mode: int, rows: torch.Tensor, p: _Plan, dst_ptrs: torch.Tensor, cap: int, ch: int,
                  src_idx: torch.Tensor | None = None) -> None:
        e = _ext.ext()
        ep = self._next()
        e.ep_transfer(mode, rows, p.C, self.rank, p.dst_start, p.offsets, p.blk_pos, p.blk_src, p.totals, dst_ptrs, cap,
                      self.flag_ptrs, self.flags, ch, ep, self.ticket, self.timeout_ns, self.status, self.ctas, src_idx)
        e.tp_wait(self.flags, ch, self._all(), ep, self.timeout_ns, self.status)

    def to_owners(self, rows: torch.Tensor, p: _Plan, which: str, src_idx: torch.Tensor | None = None) -> torch.Tensor:
        """Source-sorted rows (n_send, H) -> this rank's owner layout (n_recv, H), a fresh tensor.  With
        ``src_idx``, ``rows`` are token rows and sorted row r is ``rows[src_idx[r]]`` (gathered in the
        transfer kernel)."""
        buf, ptrs, ch = (self.recv_a, self.recv_a_ptrs, CH_A_RECV) if which == "a" else (self.recv_b, self.recv_b_ptrs, CH_B_RECV)
        self._transfer(0, rows.contiguous(), p, ptrs, self.cap_recv, ch, src_idx)
        return buf[:p.n_recv * self.hidden].view(p.n_recv, self.hidden).clone()

    def to_sources(self, rows: torch.Tensor, p: _Plan, which: str) -> torch.Tensor:
        """Owner-layout rows (n_recv, H) -> this rank's source-sorted rows (n_send, H)."""
        buf, ptrs, ch = (self.back_a, self.back_a_ptrs, CH_A_BACK) if which == "a" else (self.back_b, self.back_b_ptrs, CH_B_BACK)
        self._transfer(1, rows.contiguous(), p, ptrs, self.max_rows, ch)
        return buf[:p.n_send * self.hidden].view(p.n_send, self.hidden).clone()


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_sorted, comm, plan):  # noqa: ANN001, ANN205
        ctx.comm, ctx.plan = comm, plan
        return comm.to_owners(x_sorted, plan, "a")

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return ctx.comm.to_sources(g, ctx.plan, "b"), None, None


class _DispatchTokens(torch.autograd.Function):
    """Dispatch of token rows ``x`` (T, H) in the expert-sorted order ``order`` (flat slot t k + j),
    gathered inside the transfer kernel; the backward brings the row gradients back to the sources
    and sums each token's k slots."""

    @staticmethod
    def forward(ctx, x, order, k, comm, plan):  # noqa: ANN001, ANN205
        ctx.comm, ctx.plan, ctx.k = comm, plan, k
        ctx.save_for_backward(order)
        ctx.T = x.shape[0]
        return comm.to_owners(x, plan, "a", src_idx=(order // k).contiguous())

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        from axrl_b200.ops.grouped import moe_combine

        (order,) = ctx.saved_tensors
        g_sorted = ctx.comm.to_sources(g, ctx.plan, "b")
        ones = torch.ones(ctx.T, ctx.k, dtype=torch.float32, device=g.device)
        return moe_combine(g_sorted, ones, order), None, None, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_owner, comm, plan):  # noqa: ANN001, ANN205
        ctx.comm, ctx.plan = comm, plan
        return comm.to_sources(y_owner, plan, "a")

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return ctx.comm.to_owners(g, ctx.plan, "b"), None, None


def p2p_moe_forward(block, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, comm: P2PEPComm) -> torch.Tensor:  # noqa: ANN001
    from axrl_b200.ops.grouped import grouped_swiglu_ffn

    T, H = x.shape
    k = ids.shape[1]
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    plan = comm.plan(flat[order])
    xr = _DispatchTokens.apply(x, order, k, comm, plan)
    y = grouped_swiglu_ffn(xr, plan.offsets, block.experts_gate_up, block.experts_down)
    yb = _Combine.apply(y, comm, plan)
    from axrl_b200.ops.grouped import moe_combine

    return moe_combine(yb, w, order).to(x.dtype)

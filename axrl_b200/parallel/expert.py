"""Expert parallelism for MoE layers: token dispatch to the ranks that own the chosen experts, a
grouped expert FFN on each rank, and the combine back to the source tokens.

Reference: ``ep_size`` / ``etp_size`` (``axrl/configs.py:383-384``) with Megatron's
``moe_token_dispatcher_type="alltoall"`` (``axrl/worker/megatron_worker.py:833``) and routing
replay feeding the router (``axrl/utils/megatron/router_replay.py:67-108``).

Layout: with ``P`` EP ranks and ``E`` experts, rank ``r`` owns experts ``[r*E/P, (r+1)*E/P)``;
its MoE block holds only those experts' weights.  The router is replicated (its gradient is
reduced with the dense parameters); expert weights carry ``expert_parallel = True`` so the
trainer keeps their gradients out of the data-parallel reduction.

Two transports:

* :class:`TorchEPComm` – ``all_to_all_single`` (NCCL / gloo) with host-known split sizes (the
  baseline; one host sync per layer for the counts);
* :class:`axrl_b200.parallel.ep_p2p.P2PEPComm` – device-side dispatch/combine kernels writing rows
  straight into the owner's symmetric receive buffer over NVLink (no host sync).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist


@dataclass
class EPContext:
    size: int = 1
    rank: int = 0
    group: Any = None
    comm: Any = None
    # expert tensor parallelism: every expert's FFN columns split over ``etp_size`` ranks that hold
    # the same experts (Megatron ``expert_tensor_parallel_size``); 1 = whole experts
    etp_size: int = 1
    etp_rank: int = 0
    etp_group: Any = None

    @property
    def enabled(self) -> bool:
        return self.size > 1

    @property
    def active(self) -> bool:
        """Expert weights are split over ranks (EP and/or ETP)."""
        return self.size > 1 or self.etp_size > 1

    @classmethod
    def from_group(cls, group: Any, backend: str = "torch", etp_group: Any = None, **p2p_kw: Any) -> "EPContext":
        """``p2p_kw`` sizes the NVLink buffers (hidden, num_experts, max_rows, cap_factor)."""
        etp = dict(etp_size=dist.get_world_size(etp_group), etp_rank=dist.get_rank(etp_group), etp_group=etp_group) \
            if etp_group is not None and dist.get_world_size(etp_group) > 1 else {}
        if group is None or dist.get_world_size(group) == 1:
            return cls(**etp)
        size, rank = dist.get_world_size(group), dist.get_rank(group)
        if etp and backend == "p2p":
            raise ValueError("expert tensor parallelism runs on the NCCL transport (backend='torch')")
        if backend == "p2p":
            from axrl_b200.parallel.ep_p2p import P2PEPComm

            comm: Any = P2PEPComm(group, **p2p_kw)
        else:
            comm = TorchEPComm(group)
        return cls(size=size, rank=rank, group=group, comm=comm, **etp)


class _AllToAll(torch.autograd.Function):
    """Rows of ``x`` split by ``send`` counts to each rank; receives ``recv`` counts."""

    @staticmethod
    def forward(ctx, x, send, recv, group):  # noqa: ANN001, ANN205
        ctx.send, ctx.recv, ctx.group = send, recv, group
        out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=group)
        return out

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


class TorchEPComm:
    def __init__(self, group: Any) -> None:
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def counts(self, send_counts: torch.Tensor) -> tuple[list[int], list[int]]:
        recv = torch.empty_like(send_counts)
        dist.all_to_all_single(recv, send_counts.contiguous(), group=self.group)
        return send_counts.tolist(), recv.tolist()

    def dispatch(self, x_sorted: torch.Tensor, expert_sorted: torch.Tensor, send_counts: torch.Tensor):  # noqa: ANN201
        """Rows sorted by global expert -> (rows received, their global expert ids, context)."""
        send, recv = self.counts(send_counts)
        xr = _AllToAll.apply(x_sorted, send, recv, self.group)
        er = expert_sorted.new_empty(sum(recv))
        dist.all_to_all_single(er, expert_sorted.contiguous(), recv, send, group=self.group)
        return xr, er, (send, recv)

    def combine(self, y_recv_order: torch.Tensor, handle) -> torch.Tensor:  # noqa: ANN001
        send, recv = handle
        return _AllToAll.apply(y_recv_order, recv, send, self.group)


class _ETPGather(torch.autograd.Function):
    """Rows of every ETP rank concatenated in rank order (variable counts); backward sums the row
    gradients over the ETP ranks and keeps this rank's rows."""

    @staticmethod
    def forward(ctx, x, counts, rank, group):  # noqa: ANN001, ANN205
        ctx.counts, ctx.rank, ctx.group = counts, rank, group
        mx = max(counts)
        pad = x.new_zeros((mx,) + tuple(x.shape[1:]))
        pad[:x.shape[0]] = x
        parts = [torch.empty_like(pad) for _ in counts]
        dist.all_gather(parts, pad.contiguous(), group=group)
        return torch.cat([p[:c] for p, c in zip(parts, counts)])

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        o = sum(ctx.counts[:ctx.rank])
        return g[o:o + ctx.counts[ctx.rank]], None, None, None


class _ETPReduceScatter(torch.autograd.Function):
    """Partial rows of every ETP rank's tokens (concatenated in rank order) summed over the ETP
    ranks; this rank keeps its own rows.  Backward gathers the row gradients."""

    @staticmethod
    def forward(ctx, y, counts, rank, group):  # noqa: ANN001, ANN205
        ctx.counts, ctx.rank, ctx.group = counts, rank, group
        y = y.contiguous().clone()
        dist.all_reduce(y, group=group)
        o = sum(counts[:rank])
        return y[o:o + counts[rank]]

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _ETPGather.apply(g, ctx.counts, ctx.rank, ctx.group), None, None, None


def _etp_counts(n: int, ep: EPContext, device) -> list[int]:  # noqa: ANN001
    c = torch.tensor([n], dtype=torch.int64, device=device)
    out = [torch.empty_like(c) for _ in range(ep.etp_size)]
    dist.all_gather(out, c, group=ep.etp_group)
    return [int(t) for t in out]


def ep_moe_forward(block, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ep: EPContext) -> torch.Tensor:  # noqa: ANN001
    """MoE FFN of ``block`` (holding experts of this EP rank) for local tokens ``x`` (T, H) routed to
    global experts ``ids`` (T, k) with weights ``w`` (T, k)."""
    from axrl_b200.ops.grouped import expert_offsets, grouped_swiglu_ffn

    if hasattr(ep.comm, "plan"):  # NVLink transport: device-side plan, no host sync
        from axrl_b200.parallel.ep_p2p import p2p_moe_forward

        return p2p_moe_forward(block, x, w, ids, ep.comm)
    T, H = x.shape
    k = ids.shape[1]
    E_l = block.experts_gate_up.shape[0]
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    tok = order // k
    exp_sorted = flat[order]
    if ep.size > 1:
        send_counts = torch.bincount(exp_sorted // E_l, minlength=ep.size)
        xr, er, handle = ep.comm.dispatch(x.index_select(0, tok), exp_sorted, send_counts)
    else:  # expert tensor parallelism only: every rank holds (column shards of) all experts
        xr, er, handle = x.index_select(0, tok), exp_sorted, None
    local = er - ep.rank * E_l
    if ep.etp_size > 1:  # every ETP rank computes its FFN columns for the rows of all ETP ranks
        counts = _etp_counts(int(xr.shape[0]), ep, x.device)
        xr = _ETPGather.apply(xr, counts, ep.etp_rank, ep.etp_group)
        lg = [torch.empty(max(counts), dtype=local.dtype, device=local.device) for _ in counts]
        lp = local.new_zeros(max(counts))
        lp[:local.numel()] = local
        dist.all_gather(lg, lp, group=ep.etp_group)
        local = torch.cat([t[:c] for t, c in zip(lg, counts)])
    order2 = torch.argsort(local, stable=True)
    offsets = expert_offsets(local[order2], E_l)
    y = grouped_swiglu_ffn(xr.index_select(0, order2), offsets, block.experts_gate_up, block.experts_down)
    inv2 = torch.empty_like(order2)
    inv2[order2] = torch.arange(order2.numel(), device=order2.device)
    y = y.index_select(0, inv2)
    if ep.etp_size > 1:  # partial sums over the FFN columns -> this rank's rows
        y = _ETPReduceScatter.apply(y, counts, ep.etp_rank, ep.etp_group)
    yb = ep.comm.combine(y, handle) if handle is not None else y
    from axrl_b200.ops.grouped import moe_combine

    return moe_combine(yb, w, order).to(x.dtype)


# ----------------------------------------------------------------------------- params


def expert_params(model: torch.nn.Module) -> list[torch.nn.Parameter]:
    return [p for p in model.parameters() if getattr(p, "expert_parallel", False)]


@torch.no_grad()
def load_ep_shards_from_full(model: torch.nn.Module, full_state: dict[str, torch.Tensor], ep: EPContext) -> None:
    """Fill an EP model (local experts only) from a full (EP=1) ``named_parameters`` state."""
    for name, p in model.named_parameters():
        src = full_state[name]
        if getattr(p, "expert_parallel", False):
            E_l = p.shape[0]
            src = src[ep.rank * E_l:(ep.rank + 1) * E_l]
            if ep.etp_size > 1:  # this rank's FFN columns: gate and up halves / down columns
                r = ep.etp_rank
                if name.endswith("experts_gate_up"):
                    F = src.shape[1] // 2
                    Fl = F // ep.etp_size
                    src = torch.cat([src[:, r * Fl:(r + 1) * Fl], src[:, F + r * Fl:F + (r + 1) * Fl]], 1)
                else:
                    Fl = src.shape[2] // ep.etp_size
                    src = src[:, :, r * Fl:(r + 1) * Fl]
        p.copy_(src.to(p.device, p.dtype))


def dense_grad_allreduce(model: torch.nn.Module, group: Any) -> None:
    """All-reduce the gradients of every non-expert parameter over ``group`` (one coalesced call)."""
    ps = [p for p in model.parameters() if not getattr(p, "expert_parallel", False) and getattr(p, "main_grad", None) is not None]
    if not ps:
        return
    flat = torch.cat([p.main_grad.reshape(-1) for p in ps])
    dist.all_reduce(flat, group=group)
    off = 0
    for p in ps:
        n = p.numel()
        p.main_grad.copy_(flat[off:off + n].view(p.shape))
        off += n

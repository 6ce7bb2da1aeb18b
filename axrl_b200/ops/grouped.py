"""Grouped expert FFN over tokens sorted by expert.

Tokens arrive sorted by expert id with DEVICE row offsets (``offsets[e]:offsets[e+1]`` are expert
``e``'s rows); each expert applies ``down(swiglu(gate_up(x)))``.  On the GPU each projection is
ONE grouped tcgen05 GEMM over all experts (``csrc/kernels/grouped_gemm.cu``), so routing never
forces a host sync; backward runs the grouped dgrad and accumulates the grouped weight gradient
into the expert weights' fp32 ``main_grad``.  The CPU path loops over experts (the oracle).

Reference counterpart: Megatron's grouped expert MLP (TE grouped GEMM) used by the Qwen3-MoE
models (``axrl/worker/megatron_worker.py:833``).
"""

from __future__ import annotations

import torch

from axrl_b200.ops import _ext
from axrl_b200.ops import core as ops


class _GroupedLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, offsets):  # noqa: ANN001, ANN205
        ctx.save_for_backward(x, w, offsets)
        return _ext.ext().grouped_linear_fwd(x, w, offsets)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x, w, offsets = ctx.saved_tensors
        dy = dy.contiguous()
        e = _ext.ext()
        dx = e.grouped_linear_dgrad(dy, w, offsets) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                e.grouped_linear_wgrad_acc(dy, x, offsets, main)
            else:
                acc = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
                e.grouped_linear_wgrad_acc(dy, x, offsets, acc)
                dw = acc.to(w.dtype)
        return dx, dw, None


def grouped_linear_ref(x: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    off = offsets.tolist()
    outs = [x[off[e]:off[e + 1]] @ w[e].t() for e in range(w.shape[0])]
    return torch.cat(outs, 0) if outs else x[:0, :0]


def grouped_linear(x: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """Rows ``offsets[e]:offsets[e+1]`` of ``x`` times ``w[e].T`` for every expert ``e``."""
    if not x.is_cuda:
        return grouped_linear_ref(x, w, offsets)
    return _GroupedLinear.apply(x.contiguous(), w, offsets.to(torch.int32).contiguous())


def expert_offsets(expert_ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """(E+1,) int32 row offsets of each expert in the expert-sorted order (device, no sync)."""
    # scatter_add instead of bincount: fixed output size, so no host sync (CUDA-graph capturable)
    counts = torch.zeros(num_experts, dtype=torch.int64, device=expert_ids.device)
    counts.scatter_add_(0, expert_ids.long(), torch.ones_like(expert_ids, dtype=torch.int64))
    return torch.cat([counts.new_zeros(1), counts.cumsum(0)]).to(torch.int32)


def grouped_swiglu_ffn(x_sorted: torch.Tensor, offsets: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    return grouped_linear(ops.swiglu(grouped_linear(x_sorted, w_gate_up, offsets)), w_down, offsets)


class _MoECombine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w, pos):  # noqa: ANN001, ANN205
        ctx.save_for_backward(y, w, pos)
        return _ext.ext().moe_combine(y, w, pos)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        y, w, pos = ctx.saved_tensors
        dy, dw = _ext.ext().moe_combine_bwd(y, w, pos, g.contiguous())
        return dy, dw, None


def moe_combine(y_sorted: torch.Tensor, w: torch.Tensor, order: torch.Tensor) -> torch.Tensor:
    """(T, H) = sum over each token's k slots of ``w[t, j]`` times its expert output row.

    ``y_sorted`` row i is the output for flat slot ``order[i]`` (= t k + j), i.e. rows in the
    expert-sorted order; the sum is taken in fp32."""
    T, k = w.shape
    if not y_sorted.is_cuda:
        tok = order // k
        ys = y_sorted.float() * w.reshape(-1)[order][:, None]
        return torch.zeros(T, y_sorted.shape[1], dtype=torch.float32, device=y_sorted.device).index_add_(0, tok, ys).to(y_sorted.dtype)
    pos = torch.empty_like(order, dtype=torch.int32)
    pos[order] = torch.arange(order.numel(), device=order.device, dtype=torch.int32)
    return _MoECombine.apply(y_sorted.contiguous(), w.float().contiguous(), pos)

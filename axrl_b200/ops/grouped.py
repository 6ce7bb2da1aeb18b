"""Grouped expert FFN over tokens sorted by expert.

Tokens arrive sorted by expert id with per-expert counts; each expert applies
``down(swiglu(gate_up(x)))``.  This first version issues one tcgen05 GEMM pair per
non-empty expert (the same kernels as the dense layers, so numerics and autograd are
shared); the expert-parallel path (:mod:`axrl_b200.parallel.expert`) feeds it the tokens
received from peers.
"""

from __future__ import annotations

import torch

from axrl_b200.ops import core as ops


def grouped_swiglu_ffn(x_sorted: torch.Tensor, counts: list[int], w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    outs = []
    s = 0
    for e, c in enumerate(counts):
        if c:
            xe = x_sorted[s:s + c]
            outs.append(ops.linear(ops.swiglu(ops.linear(xe, w_gate_up[e])), w_down[e]))
        s += c
    return torch.cat(outs, 0) if outs else x_sorted[:0]

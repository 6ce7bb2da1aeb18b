"""Sparse MoE block (Qwen3-MoE): fp32 router, top-k softmax routing, SwiGLU experts.

Routing replay (R3, reference ``axrl/utils/megatron/router_replay.py:67-108``):
when ``ctx.replay[layer]`` holds top-k expert ids recorded by the rollout
engine, the forward uses those ids (recomputing only the gate weights from the
current router logits); with ``ctx.loss_tokens_only`` the replayed ids apply
on loss tokens and the live top-k elsewhere.  ``ctx.capture`` collects the ids
actually used, per layer, which is how the rollout engine records routing.

On a single GPU the expert FFNs run as one grouped GEMM over tokens sorted by
expert; under expert parallelism :mod:`axrl_b200.parallel.expert` replaces the
local dispatch with the fused all-to-all path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

from axrl_b200.ops import core as ops
from axrl_b200.ops.grouped import expert_offsets, grouped_swiglu_ffn, moe_combine


@dataclass
class MoEContext:
    replay: dict[int, torch.Tensor] | None = None  # layer -> (T, K) int
    replay_mask: torch.Tensor | None = None  # (T,) bool, replay only where True
    capture: dict[int, torch.Tensor] | None = None  # filled with (T, K) int16
    aux_loss: list[torch.Tensor] = field(default_factory=list)

    def rows(self, a: int, b: int) -> "MoEContext":
        """The context for token rows [a, b) (the sequence-parallel slice of a TP rank)."""
        return MoEContext(replay={k: v[a:b] for k, v in self.replay.items()} if self.replay else self.replay,
                          replay_mask=self.replay_mask[a:b] if self.replay_mask is not None else None,
                          capture=self.capture, aux_loss=self.aux_loss)


class _RouterLinear(torch.autograd.Function):
    """fp32 router logits; the weight gradient goes straight into ``main_grad`` when present."""

    @staticmethod
    def forward(ctx, x, w):  # noqa: ANN001, ANN205
        ctx.save_for_backward(x, w)
        return torch.nn.functional.linear(x.float(), w.float())

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        x, w = ctx.saved_tensors
        dx = (g @ w.float()).to(x.dtype)
        dw = g.t() @ x.float()
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.add_(dw)
            return dx, None
        return dx, dw.to(w.dtype)


def router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return _RouterLinear.apply(x, w)


class _FusedRoute(torch.autograd.Function):
    """Softmax + top-k (or replayed ids) + renormalisation in one kernel; the backward goes
    through the selected probabilities and the softmax."""

    @staticmethod
    def forward(ctx, logits, k, renorm, replay, replay_mask):  # noqa: ANN001, ANN205
        from axrl_b200.ops import _ext

        w, ids, probs = _ext.ext().router_topk(logits.contiguous(), k, renorm, replay, replay_mask)
        ctx.save_for_backward(probs, ids, w)
        ctx.renorm = renorm
        ctx.mark_non_differentiable(ids)
        return w, ids

    @staticmethod
    def backward(ctx, g_w, _g_ids):  # noqa: ANN001, ANN205
        probs, ids, w = ctx.saved_tensors
        g = g_w.float()
        if ctx.renorm:  # w = p_sel / S:  dp_sel = (g - sum(g * w)) / S
            p_sel = probs.gather(1, ids)
            S = p_sel.sum(-1, keepdim=True).clamp_min(1e-20)
            g = (g - (g * w).sum(-1, keepdim=True)) / S
        dprobs = torch.zeros_like(probs).scatter_add_(1, ids, g)
        dlogits = probs * (dprobs - (dprobs * probs).sum(-1, keepdim=True))
        return dlogits, None, None, None, None


def route(logits: torch.Tensor, k: int, renorm: bool, replay: torch.Tensor | None = None, replay_mask: torch.Tensor | None = None):  # noqa: ANN201
    """Top-k routing in fp32.  Returns (weights (T,k) fp32, ids (T,k) int64)."""
    if logits.is_cuda and k <= 8 and logits.shape[-1] <= 256:
        return _FusedRoute.apply(logits.float(), int(k), bool(renorm), None if replay is None else replay.long().contiguous(),
                                 None if replay_mask is None or replay is None else replay_mask.bool().contiguous())
    probs = torch.softmax(logits.float(), -1)
    top_w, top_i = probs.topk(k, -1)
    if replay is not None:
        rep = replay.long()
        if replay_mask is not None:
            rep = torch.where(replay_mask[:, None], rep, top_i)
        top_i = rep
        top_w = probs.gather(1, top_i)
    if renorm:
        top_w = top_w / top_w.sum(-1, keepdim=True).clamp_min(1e-20)
    return top_w, top_i


def grouped_ffn_ref(x_sorted: torch.Tensor, counts: list[int], w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    outs, s = [], 0
    for e, c in enumerate(counts):
        if c:
            xe = x_sorted[s:s + c]
            outs.append(ops.linear(ops.swiglu(ops.linear(xe, w_gate_up[e])), w_down[e]))
        s += c
    return torch.cat(outs, 0) if outs else x_sorted[:0]


class MoEBlock(nn.Module):
    def __init__(self, cfg, ep=None) -> None:  # noqa: ANN001
        super().__init__()
        E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        self.E, self.k, self.renorm = E, cfg.num_experts_per_tok, cfg.norm_topk_prob
        self.ep = ep
        ep_size = ep.size if ep is not None else 1
        etp = ep.etp_size if ep is not None else 1
        assert E % ep_size == 0, "experts must split evenly over EP ranks"
        assert F % etp == 0, "expert FFN width must split evenly over expert-TP ranks"
        E_l, F_l = E // ep_size, F // etp  # experts held by this rank, and their FFN columns
        self.router = nn.Parameter(torch.empty(E, H))
        self.experts_gate_up = nn.Parameter(torch.empty(E_l, 2 * F_l, H))
        self.experts_down = nn.Parameter(torch.empty(E_l, H, F_l))
        if ep_size > 1 or etp > 1:
            self.experts_gate_up.expert_parallel = True
            self.experts_down.expert_parallel = True
        # shared expert (Qwen3-Next / 3.5): a dense SwiGLU FFN every token passes through, scaled by
        # sigmoid(x . shared_gate); replicated like the attention weights, not expert-parallel
        Fs = getattr(cfg, "shared_expert_intermediate_size", 0)
        self.shared_gate_up = nn.Parameter(torch.empty(2 * Fs, H)) if Fs else None
        self.shared_down = nn.Parameter(torch.empty(H, Fs)) if Fs else None
        self.shared_gate = nn.Parameter(torch.empty(1, H)) if Fs else None

    def shared_expert(self, x: torch.Tensor, linear=None) -> torch.Tensor | None:  # noqa: ANN001
        """Gated shared-expert output for ``x`` (T, H) (None without a shared expert)."""
        if self.shared_gate_up is None:
            return None
        lin = linear or ops.linear
        y = lin(ops.swiglu(lin(x, self.shared_gate_up)), self.shared_down)
        # the (T, 1) gate logit is a matrix-vector product: fp32, outside the tiled GEMM kernels
        gate = torch.nn.functional.linear(x.float(), self.shared_gate.float())
        return y * torch.sigmoid(gate).to(y.dtype)

    def hf_tensors(self, prefix: str) -> dict[str, torch.Tensor]:
        out = {prefix + "mlp.gate.weight": self.router}
        if self.shared_gate_up is not None:
            g, u = self.shared_gate_up.chunk(2, 0)
            out |= {prefix + "mlp.shared_expert.gate_proj.weight": g, prefix + "mlp.shared_expert.up_proj.weight": u,
                    prefix + "mlp.shared_expert.down_proj.weight": self.shared_down,
                    prefix + "mlp.shared_expert_gate.weight": self.shared_gate}
        F = self.experts_down.shape[2]
        for e in range(self.E):
            q = f"{prefix}mlp.experts.{e}."
            out[q + "gate_proj.weight"] = self.experts_gate_up[e, :F]
            out[q + "up_proj.weight"] = self.experts_gate_up[e, F:]
            out[q + "down_proj.weight"] = self.experts_down[e]
        return out

    shared_selective = False  # selective recompute of the shared expert (recompute_modules)

    def forward(self, x: torch.Tensor, ctx: MoEContext | None = None, layer_idx: int = 0) -> torch.Tensor:
        y = self._routed(x, ctx, layer_idx)
        if self.shared_selective and torch.is_grad_enabled():  # recompute the shared expert in backward
            from torch.utils.checkpoint import checkpoint

            sh = checkpoint(self.shared_expert, x, use_reentrant=False)
        else:
            sh = self.shared_expert(x)
        return y if sh is None else y + sh

    def _routed(self, x: torch.Tensor, ctx: MoEContext | None, layer_idx: int) -> torch.Tensor:
        T, H = x.shape
        logits = router_logits(x, self.router)
        replay = ctx.replay.get(layer_idx) if ctx is not None and ctx.replay else None
        w, ids = route(logits, self.k, self.renorm, replay, ctx.replay_mask if ctx is not None else None)
        if ctx is not None and ctx.capture is not None:
            ctx.capture[layer_idx] = ids.to(torch.int16)
        if self.ep is not None and (self.ep.enabled or self.ep.etp_size > 1):
            from axrl_b200.parallel.expert import ep_moe_forward

            return ep_moe_forward(self, x, w, ids, self.ep)
        flat = ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        tok = order // self.k
        offsets = expert_offsets(flat, self.E)
        xs = x.index_select(0, tok)
        ys = grouped_swiglu_ffn(xs, offsets, self.experts_gate_up, self.experts_down)
        return moe_combine(ys, w, order).to(x.dtype)

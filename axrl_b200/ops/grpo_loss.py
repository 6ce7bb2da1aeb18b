"""Fused GRPO / PPO clipped policy objective (``csrc/kernels/grpo_loss.cu``).

One kernel evaluates, per token, the importance ratio, the PPO clip, the dual clip on negative
advantages and the truncated-IS / mask weight, and writes the per-token loss together with its
gradient w.r.t. the current log-probs; the backward is a single scale.  Semantics are those of
:meth:`axrl_b200.trainer.grpo_trainer.GrpoTrainer.grpo_loss` (reference
``axrl/trainer/grpo_trainer.py:197-803``), which remains the CPU path and the test oracle.
"""

from __future__ import annotations

import torch

from axrl_b200.ops import _ext


class _GrpoPG(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lp, base, adv, w, lo, hi, dual):  # noqa: ANN001, ANN205
        out, grad, ratio, eff = _ext.ext().grpo_pg_fwd(lp.contiguous(), base.contiguous(), adv.contiguous(), w.contiguous(), lo, hi, dual)
        ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(ratio, eff)
        return out, ratio, eff

    @staticmethod
    def backward(ctx, g, _gr, _ge):  # noqa: ANN001, ANN205
        (grad,) = ctx.saved_tensors
        return _ext.ext().grpo_pg_bwd(g.float(), grad), None, None, None, None, None, None


def grpo_policy_loss(logprobs: torch.Tensor, base: torch.Tensor, adv: torch.Tensor, weight: torch.Tensor, clip_low: float,
                     clip_high: float, dual_clip: float | None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-token ``pg * weight`` (differentiable in ``logprobs``), the ratio and the effective ratio."""
    f = lambda t: t.float()  # noqa: E731
    return _GrpoPG.apply(f(logprobs), f(base).detach(), f(adv).detach(), f(weight).detach(), float(clip_low), float(clip_high),
                         float(dual_clip) if dual_clip is not None else 0.0)

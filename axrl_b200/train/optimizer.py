"""Flat-buffer AdamW with fp32 master weights (the single-rank core of the distributed optimizer).

Reference counterpart: Megatron's distributed optimizer with fused Adam, fp32
grad buffers (``grad_reduce_in_fp32``) and global-norm clipping
(``axrl/worker/megatron_worker.py:480-509,905-930``; config
``axrl/configs.py:309-334``).

Layout: every parameter's bf16 storage is a view into ONE flat bf16 buffer;
fp32 master weights, Adam moments and fp32 gradients are flat buffers of the
same element order (weight-decayed params first, then norms/biases).  Each
parameter gets ``p.main_grad`` (a view into the grad buffer) that the
weight-gradient GEMMs accumulate into directly.  One kernel computes the
squared norm, one fused kernel clips + updates + writes the bf16 params back:
no per-parameter launches and no host synchronisation.

The grad buffer can be dropped between steps (:meth:`release_grads`) to make
room for the rollout engine's KV cache when both share a GPU.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig
from axrl_b200.ops import _ext


def lr_at(step: int, c: MCoreLrSchedulerConfig) -> float:
    """Warmup from init_lr to max_lr, then constant / linear / cosine decay to min_lr."""
    if c.lr_warmup_steps > 0 and step < c.lr_warmup_steps:
        return c.init_lr + (c.max_lr - c.init_lr) * step / c.lr_warmup_steps
    if c.lr_decay_style == "constant":
        return c.max_lr
    t = min(1.0, (step - c.lr_warmup_steps) / max(1, c.lr_decay_steps - c.lr_warmup_steps))
    if c.lr_decay_style == "linear":
        return c.max_lr - (c.max_lr - c.min_lr) * t
    return c.min_lr + 0.5 * (c.max_lr - c.min_lr) * (1 + math.cos(math.pi * t))


class FlatAdamW:
    def __init__(self, model: nn.Module, opt: MCoreOptimizerConfig, sched: MCoreLrSchedulerConfig, *, shard: tuple[int, int] | None = None):
        self.opt, self.sched = opt, sched
        params = [p for p in model.parameters() if p.requires_grad]
        decay = [p for p in params if p.dim() >= 2]
        no_decay = [p for p in params if p.dim() < 2]
        self.params = decay + no_decay
        self.decay_end = sum(p.numel() for p in decay)
        self.numel = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.device = dev
        self.bf16 = torch.empty(self.numel, dtype=self.params[0].dtype, device=dev)  # parameter storage (bf16 on GPU)
        self.master = torch.empty(self.numel, dtype=torch.float32, device=dev)
        off = 0
        self.offsets = []
        for p in self.params:
            n = p.numel()
            self.master[off:off + n].copy_(p.detach().reshape(-1).float())
            self.bf16[off:off + n].copy_(p.detach().reshape(-1))
            p.data = self.bf16[off:off + n].view(p.shape)
            self.offsets.append(off)
            off += n
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.grad: torch.Tensor | None = None
        self.step_count = 0
        self.alloc_grads()
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)

    # -------------------------------------------------------------- grads
    def alloc_grads(self) -> None:
        if self.grad is None:
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        for p, off in zip(self.params, self.offsets):
            p.main_grad = self.grad[off:off + p.numel()].view(p.shape)

    def release_grads(self) -> None:
        for p in self.params:
            if hasattr(p, "main_grad"):
                del p.main_grad
        self.grad = None

    def zero_grad(self) -> None:
        self.alloc_grads()
        self.grad.zero_()
        for p in self.params:
            p.grad = None

    def fold_param_grads(self) -> None:
        """Add any autograd ``.grad`` (ops that do not write main_grad) into the flat buffer."""
        for p in self.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None

    # -------------------------------------------------------------- step
    def grad_sqnorm(self, scale: float = 1.0) -> torch.Tensor:
        """Device scalar ``sum(grad^2)`` of the unscaled buffer (no host sync)."""
        self._sq.zero_()
        if self.grad.is_cuda:
            _ext.ext().sqnorm_accumulate(self.grad, self._sq)
        else:
            self._sq += self.grad.double().square().sum().float()
        return self._sq

    def step(self, grad_scale: float = 1.0, sqnorm: torch.Tensor | None = None) -> torch.Tensor:
        """Clip by global norm (from ``sqnorm`` of the unscaled grads, times grad_scale),
        AdamW update, write bf16 params.  Returns the (device) grad norm after scaling."""
        self.fold_param_grads()
        self.step_count += 1
        o = self.opt
        lr = lr_at(self.step_count - 1, self.sched)
        wd = o.weight_decay
        if sqnorm is None:
            sqnorm = self.grad_sqnorm()
        norm = sqnorm.sqrt() * grad_scale
        if self.grad.is_cuda:
            _ext.ext().adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.bf16, self.decay_end, lr,
                                  o.adam_beta1, o.adam_beta2, o.adam_eps, wd, self.step_count, sqnorm, float(o.clip_grad),
                                  float(grad_scale))
        else:
            self._cpu_step(lr, grad_scale, norm)
        return norm

    def _cpu_step(self, lr: float, grad_scale: float, norm: torch.Tensor) -> None:
        o = self.opt
        g = self.grad * grad_scale
        if o.clip_grad > 0:
            g = g * torch.clamp(o.clip_grad / (norm + 1e-6), max=1.0)
        b1, b2 = o.adam_beta1, o.adam_beta2
        self.exp_avg.mul_(b1).add_(g, alpha=1 - b1)
        self.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        upd = (self.exp_avg / bc1) / ((self.exp_avg_sq / bc2).sqrt() + o.adam_eps)
        upd[: self.decay_end] += o.weight_decay * self.master[: self.decay_end]
        self.master.add_(upd, alpha=-lr)
        self.bf16.copy_(self.master)

    # -------------------------------------------------------------- state
    def state_dict(self) -> dict:
        return {"master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq, "step": self.step_count}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.step_count = int(sd["step"])
        self.bf16.copy_(self.master)

    @torch.no_grad()
    def sync_master_from_params(self) -> None:
        """After loading weights into the bf16 params, refresh the fp32 masters."""
        self.master.copy_(self.bf16.float())

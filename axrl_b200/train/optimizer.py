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
room for the rollout engine's KV cache when both share a GPU.  With
``optimizer_cpu_offload`` the tail ``optimizer_offload_fraction`` of the fp32
state lives in pinned host memory and is updated on the CPU
(:class:`axrl_b200.train.offload.AdamState`).
"""

from __future__ import annotations

import math

import torch
from torch import nn

from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig
from axrl_b200.ops import _ext
from axrl_b200.train.offload import AdamState, offload_fraction


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
        master = torch.empty(self.numel, dtype=torch.float32, device=dev)
        off = 0
        self.offsets = []
        for p in self.params:
            n = p.numel()
            master[off:off + n].copy_(p.detach().reshape(-1).float())
            self.bf16[off:off + n].copy_(p.detach().reshape(-1))
            p.data = self.bf16[off:off + n].view(p.shape)
            self.offsets.append(off)
            off += n
        self.state = AdamState(master, offload_fraction(opt))
        del master
        self.grad: torch.Tensor | None = None
        self.step_count = 0
        self.alloc_grads()
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)

    # device-resident state (the whole state unless part of it is offloaded to the host)
    @property
    def master(self) -> torch.Tensor:
        return self.state.dev_master

    @property
    def exp_avg(self) -> torch.Tensor:
        return self.state.dev_m

    @property
    def exp_avg_sq(self) -> torch.Tensor:
        return self.state.dev_v

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
        self.state.step_range(0, self.numel, self.grad, self.bf16, self.decay_end, lr, o, self.step_count, sqnorm, grad_scale)
        return norm

    # -------------------------------------------------------------- state
    def state_dict(self) -> dict:
        st = self.state
        return {"master": st.master_full(), "exp_avg": st.m_full(), "exp_avg_sq": st.v_full(), "step": self.step_count}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.state.load(sd["master"], sd["exp_avg"], sd["exp_avg_sq"])
        self.step_count = int(sd["step"])
        self.bf16.copy_(sd["master"].reshape(-1).to(self.bf16.device))

    @torch.no_grad()
    def sync_master_from_params(self) -> None:
        """After loading weights into the bf16 params, refresh the fp32 masters."""
        self.state.load(self.bf16.float())

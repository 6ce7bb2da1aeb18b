"""Distributed (ZeRO-1 style) AdamW over data-parallel ranks.

Reference counterpart: Megatron DDP + distributed optimizer
(``use_distributed_optimizer=True``, ``grad_reduce_in_fp32``; ``axrl/configs.py:316``,
``axrl/worker/megatron_worker.py:905-930``): fp32 grads are reduce-scattered, each DP
rank updates only its shard of the fp32 master weights / Adam moments, and the
updated bf16 parameters are all-gathered.

Two implementations of the same step:

* ``backend="nccl"`` – ``reduce_scatter_tensor`` -> local fused AdamW kernel on the
  shard -> ``all_gather_into_tensor`` of bf16 params (the baseline);
* ``backend="p2p"`` – the fused path: gradients live in a symmetric-memory buffer;
  one kernel pulls every peer's slice of this rank's shard over NVLink (P2P loads),
  sums, scales and accumulates the squared norm; after a device-side barrier a second
  kernel applies clipped AdamW to the shard and stores the new bf16 values straight
  into every peer's parameter buffer (P2P stores).  No NCCL call, no staging copies.

Memory per rank: bf16 params (full) + fp32 grads (full, reduced in place) + fp32
master/m/v for 1/N of the parameters.
"""

from __future__ import annotations


import torch
import torch.distributed as dist
from torch import nn

from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig
from axrl_b200.ops import _ext
from axrl_b200.train.optimizer import lr_at


class DistributedAdamW:
    def __init__(self, model: nn.Module, opt: MCoreOptimizerConfig, sched: MCoreLrSchedulerConfig, group=None,  # noqa: ANN001
                 backend: str = "nccl") -> None:
        self.opt, self.sched, self.group = opt, sched, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.backend = backend
        params = [p for p in model.parameters() if p.requires_grad]
        decay = [p for p in params if p.dim() >= 2]
        no_decay = [p for p in params if p.dim() < 2]
        self.params = decay + no_decay
        self.decay_end = sum(p.numel() for p in decay)
        n = sum(p.numel() for p in self.params)
        self.numel = n
        align = self.world * 64
        self.padded = -(-n // align) * align
        self.shard = self.padded // self.world
        self.s0 = self.rank * self.shard
        dev = self.params[0].device
        self.device = dev
        symm = backend == "p2p"
        if symm:
            import torch.distributed._symmetric_memory as symm_mem

            self._symm = symm_mem
            self.bf16 = symm_mem.empty(self.padded, dtype=self.params[0].dtype, device=dev)
            self.grad = symm_mem.empty(self.padded, dtype=torch.float32, device=dev)
            gname = (group or dist.group.WORLD).group_name
            self.h_param = symm_mem.rendezvous(self.bf16, gname)
            self.h_grad = symm_mem.rendezvous(self.grad, gname)
            self.param_ptrs = torch.tensor(self.h_param.buffer_ptrs, dtype=torch.int64, device=dev)
            self.grad_ptrs = torch.tensor(self.h_grad.buffer_ptrs, dtype=torch.int64, device=dev)
        else:
            self.bf16 = torch.zeros(self.padded, dtype=self.params[0].dtype, device=dev)
            self.grad = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        self.bf16.zero_()
        off = 0
        self.offsets = []
        for p in self.params:
            k = p.numel()
            self.bf16[off:off + k].copy_(p.detach().reshape(-1))
            p.data = self.bf16[off:off + k].view(p.shape)
            self.offsets.append(off)
            off += k
        self.master = self.bf16[self.s0:self.s0 + self.shard].float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.red = torch.empty(self.shard, dtype=torch.float32, device=dev) if not symm else None
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.step_count = 0
        self.attach_grads()

    def attach_grads(self) -> None:
        for p, off in zip(self.params, self.offsets):
            p.main_grad = self.grad[off:off + p.numel()].view(p.shape)

    def release_grads(self) -> None:  # grads are needed by the symmetric buffer; keep allocated
        pass

    def alloc_grads(self) -> None:
        self.attach_grads()

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p in self.params:
            p.grad = None

    def fold_param_grads(self) -> None:
        for p in self.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None

    def grad_sqnorm(self) -> torch.Tensor:
        return self._sq

    @property
    def shard_decay_end(self) -> int:
        return max(0, min(self.shard, self.decay_end - self.s0))

    def step(self, grad_scale: float = 1.0, sqnorm: torch.Tensor | None = None) -> torch.Tensor:
        """Reduce-scatter grads, clip by the global norm, AdamW on the shard, gather bf16 params."""
        self.fold_param_grads()
        self.step_count += 1
        o = self.opt
        lr = lr_at(self.step_count - 1, self.sched)
        e = _ext.ext()
        self._sq.zero_()
        if self.backend == "p2p":
            # phase 1: every rank's grads are complete before any peer reads them
            self.h_grad.barrier(channel=0)
            e.p2p_reduce_shard(self.grad_ptrs, self.grad, self.s0, self.shard, self.world, self._sq)
            dist.all_reduce(self._sq, group=self.group)
            red = self.grad[self.s0:self.s0 + self.shard]
            e.adamw_step(self.master, red, self.exp_avg, self.exp_avg_sq, None, self.shard_decay_end, lr, o.adam_beta1, o.adam_beta2,
                         o.adam_eps, o.weight_decay, self.step_count, self._sq, float(o.clip_grad), float(grad_scale))
            # phase 2: broadcast the new bf16 shard into every peer's parameter buffer
            self.h_param.barrier(channel=1)
            e.p2p_broadcast_shard(self.param_ptrs, self.master, self.s0, self.shard, self.world)
            self.h_param.barrier(channel=2)
        else:
            dist.reduce_scatter_tensor(self.red, self.grad, group=self.group)
            e.sqnorm_accumulate(self.red, self._sq)
            dist.all_reduce(self._sq, group=self.group)
            shard_bf16 = self.bf16[self.s0:self.s0 + self.shard]
            e.adamw_step(self.master, self.red, self.exp_avg, self.exp_avg_sq, shard_bf16, self.shard_decay_end, lr, o.adam_beta1,
                         o.adam_beta2, o.adam_eps, o.weight_decay, self.step_count, self._sq, float(o.clip_grad), float(grad_scale))
            dist.all_gather_into_tensor(self.bf16, shard_bf16.clone(), group=self.group)
        return self._sq.sqrt() * grad_scale

    def state_dict(self) -> dict:
        return {"master_shard": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq, "step": self.step_count,
                "shard": (self.s0, self.shard, self.numel)}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.master.copy_(sd["master_shard"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.step_count = int(sd["step"])

    @torch.no_grad()
    def sync_master_from_params(self) -> None:
        self.master.copy_(self.bf16[self.s0:self.s0 + self.shard].float())

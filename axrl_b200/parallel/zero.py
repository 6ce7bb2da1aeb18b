"""ZeRO-1 AdamW whose gradient reduce-scatter runs bucket by bucket DURING backward.

Reference counterpart: Megatron DDP with ``overlap_grad_reduce`` + the distributed optimizer
(``use_distributed_optimizer``, ``axrl/configs.py:316``; ``axrl/worker/megatron_worker.py:905-930``):
fp32 gradients are reduce-scattered in buckets as soon as backward has produced them, each DP
rank updates its shard of the fp32 master weights and Adam moments, and the new bf16 parameters
are gathered.

Layout.  Parameters are laid out in backward-completion order — final norm / LM head, then the
decoder layers from last to first, then the embedding — and cut into buckets at layer boundaries
(each at least ``bucket_elems`` elements, padded to a multiple of ``64 * world``).  Inside a bucket
the matrices come first and the vectors (norm weights, no weight decay) last, so the decayed part
of every shard is a prefix.  Rank ``r`` owns slice ``r`` of every bucket.

Overlap.  The model calls :meth:`on_layer_grads_ready` when the gradient of a layer's INPUT has
been produced during the final micro-batch's backward: every parameter of that layer (and of all
later layers) then has its final ``main_grad`` queued on the compute stream.  Buckets that became
complete are reduced on a side stream right away:

* ``backend="p2p"``: a zero-byte flag barrier over NVLink (every rank's bucket is final), then one
  kernel pulls every peer's slice of this rank's shard (P2P loads), sums it in place and
  accumulates its squared norm;
* ``backend="nccl"``: ``reduce_scatter_tensor`` of the bucket.

``step`` then all-reduces the squared norm (one float) and, per bucket, runs ONE kernel that
applies the clipped AdamW update to this rank's shard and stores the new bf16 values into every
rank's parameter buffer over NVLink (``adamw_p2p_k``: the partitioned update fused with the
parameter all-gather); with the NCCL backend the update writes the local bf16 shard and the
buckets are all-gathered.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig
from axrl_b200.ops import _ext
from axrl_b200.train.optimizer import lr_at

CH_GRAD, CH_PARAM = 7, 8


def backward_order_groups(model: nn.Module) -> list[tuple[int | None, list[nn.Parameter]]]:
    """(trigger layer, params) groups in the order backward finalises them.  The trigger is the
    global index of the layer whose input gradient completes the group (None: after backward)."""
    groups: list[tuple[int | None, list[nn.Parameter]]] = []
    layers = list(getattr(model, "layers", []))
    head = [p for p in (getattr(model, "norm", None) and model.norm.weight, getattr(model, "lm_head", None)) if p is not None]
    seen = set()
    for i, layer in enumerate(reversed(layers)):
        ps = [p for p in layer.parameters() if p.requires_grad]
        if i == 0:
            ps = head + ps
        groups.append((layer.layer_idx, ps))
        seen.update(id(p) for p in ps)
    rest = [p for p in model.parameters() if p.requires_grad and id(p) not in seen]
    if rest:
        groups.append((None, rest))
    return groups


class BucketedZeroAdamW:
    def __init__(self, model: nn.Module, opt: MCoreOptimizerConfig, sched: MCoreLrSchedulerConfig, group: Any = None,
                 backend: str = "p2p", bucket_elems: int = 64 << 20, overlap: bool = True) -> None:
        self.opt, self.sched, self.group, self.backend = opt, sched, group, backend
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        first = next(model.parameters())
        self.device = dev = first.device
        self.overlap = overlap and dev.type == "cuda"
        align = 64 * self.world
        # ---- buckets
        buckets: list[dict] = []
        cur: dict | None = None
        for trig, ps in backward_order_groups(model):
            if cur is None or cur["n"] >= bucket_elems or trig is None:
                cur = {"params": [], "n": 0, "trigger": trig}
                buckets.append(cur)
            cur["params"].extend(ps)
            cur["n"] += sum(p.numel() for p in ps)
            cur["trigger"] = trig  # completes when the LOWEST layer of the bucket is done
        off = 0
        self.params: list[nn.Parameter] = []
        self.offsets: list[int] = []
        for b in buckets:
            mats = [p for p in b["params"] if p.dim() >= 2]
            vecs = [p for p in b["params"] if p.dim() < 2]
            b["start"] = off
            b["decay_n"] = sum(p.numel() for p in mats)
            o = off
            for p in mats + vecs:
                self.params.append(p)
                self.offsets.append(o)
                o += p.numel()
            size = -(-(o - off) // align) * align
            b["size"] = size
            b["shard"] = size // self.world
            b["s0"] = off + self.rank * b["shard"]
            off += size
        self.buckets = buckets
        self.numel = off
        # ---- flat buffers (symmetric for the NVLink backend)
        if backend == "p2p":
            import torch.distributed._symmetric_memory as symm_mem

            gname = (group or dist.group.WORLD).group_name
            self.bf16 = symm_mem.empty(off, dtype=first.dtype, device=dev)
            self.grad = symm_mem.empty(off, dtype=torch.float32, device=dev)
            self.flags = symm_mem.empty(32 * 8, dtype=torch.int32, device=dev)
            self.h_param = symm_mem.rendezvous(self.bf16, gname)
            self.h_grad = symm_mem.rendezvous(self.grad, gname)
            self.h_flags = symm_mem.rendezvous(self.flags, gname)
            self.param_ptrs = torch.tensor(self.h_param.buffer_ptrs, dtype=torch.int64, device=dev)
            self.grad_ptrs = torch.tensor(self.h_grad.buffer_ptrs, dtype=torch.int64, device=dev)
            self.flag_ptrs = torch.tensor(self.h_flags.buffer_ptrs, dtype=torch.int64)
            self.flags.zero_()
            self.ticket = torch.zeros(32, dtype=torch.int32, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.epoch = 0
            self._empty = torch.zeros(16, dtype=torch.uint8, device=dev)
            self.h_flags.barrier(channel=0)
        else:
            self.bf16 = torch.zeros(off, dtype=first.dtype, device=dev)
            self.grad = torch.zeros(off, dtype=torch.float32, device=dev)
        self.bf16.zero_()
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.bf16[o:o + n].copy_(p.detach().reshape(-1))
            p.data = self.bf16[o:o + n].view(p.shape)
        # ---- my shard of every bucket: fp32 master + moments, concatenated
        self.shard_off = []
        tot = 0
        for b in buckets:
            self.shard_off.append(tot)
            tot += b["shard"]
        from axrl_b200.train.offload import AdamState, offload_fraction

        # fp32 master + moments of my shards; with optimizer_cpu_offload the tail fraction is on the host
        self.state = AdamState(torch.cat([self.bf16[b["s0"]:b["s0"] + b["shard"]].float() for b in buckets]), offload_fraction(opt))
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.step_count = 0
        self.comm_stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self._reduced: set[int] = set()
        self._armed = False
        self.timeout_ns = int(60e9)
        self.attach_grads()
        self._by_trigger: dict[int, list[int]] = {}
        for i, b in enumerate(buckets):
            if b["trigger"] is not None:
                self._by_trigger.setdefault(b["trigger"], []).append(i)
        model.grad_ready_hook = self.on_layer_grads_ready

    # -------------------------------------------------------------- grads
    def attach_grads(self) -> None:
        for p, o in zip(self.params, self.offsets):
            p.main_grad = self.grad[o:o + p.numel()].view(p.shape)

    def alloc_grads(self) -> None:
        self.attach_grads()

    def release_grads(self) -> None:
        pass  # the gradient buffer is symmetric / bucketed: kept for the next step

    def zero_grad(self) -> None:
        self.grad.zero_()
        self._sq.zero_()
        self._reduced.clear()
        for p in self.params:
            p.grad = None

    def fold_param_grads(self) -> None:
        for p in self.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None

    def arm(self, on: bool = True) -> None:
        """Enable bucket reduction from backward hooks (set before the LAST micro-batch's backward)."""
        self._armed = on and self.overlap

    def on_layer_grads_ready(self, layer_idx: int) -> None:
        if not self._armed:
            return
        for bi in self._by_trigger.get(layer_idx, []):
            self._reduce_bucket(bi)

    # -------------------------------------------------------------- reduce
    def _barrier(self, ch: int) -> None:
        self.epoch += 1
        e = _ext.ext()
        e.tp_push(self._empty, 0, 0, self.flag_ptrs, 0, self.flag_ptrs, self.flags, ch, self.epoch, self.rank,
                  (1 << self.world) - 1, self.ticket, self.timeout_ns, self.status, 1)
        e.tp_wait(self.flags, ch, ((1 << self.world) - 1) & ~(1 << self.rank), self.epoch, self.timeout_ns, self.status)

    def _reduce_bucket(self, bi: int) -> None:
        if bi in self._reduced:
            return
        self._reduced.add(bi)
        b = self.buckets[bi]
        cur = torch.cuda.current_stream() if self.comm_stream is not None else None
        if cur is not None:
            self.comm_stream.wait_stream(cur)
        ctx = torch.cuda.stream(self.comm_stream) if self.comm_stream is not None else _Null()
        with ctx:
            if self.backend == "p2p":
                self._barrier(CH_GRAD)
                _ext.ext().p2p_reduce_shard(self.grad_ptrs, self.grad, b["s0"], b["shard"], self.world, self._sq)
            else:
                red = self.grad[b["s0"]:b["s0"] + b["shard"]]
                full = self.grad[b["start"]:b["start"] + b["size"]]
                if dist.get_backend(self.group) == "nccl":
                    dist.reduce_scatter_tensor(red, full.clone(), group=self.group)
                else:  # gloo: all-reduce the bucket, keep the shard
                    dist.all_reduce(full, group=self.group)
                if red.is_cuda:
                    _ext.ext().sqnorm_accumulate(red, self._sq)
                else:
                    self._sq += red.double().square().sum().float()

    def finish_grad_sync(self) -> None:
        """Reduce every bucket not reduced during backward; wait for all reductions."""
        self._armed = False
        self.fold_param_grads()
        for bi in range(len(self.buckets)):
            self._reduce_bucket(bi)
        if self.comm_stream is not None:
            torch.cuda.current_stream().wait_stream(self.comm_stream)

    def grad_sqnorm(self) -> torch.Tensor:
        """Squared global norm of the reduced gradients (after :meth:`finish_grad_sync`)."""
        sq = self._sq.clone()
        dist.all_reduce(sq, group=self.group)
        return sq

    # -------------------------------------------------------------- step
    def step(self, grad_scale: float = 1.0, sqnorm: torch.Tensor | None = None) -> torch.Tensor:
        self.finish_grad_sync()
        if sqnorm is None:
            sqnorm = self.grad_sqnorm()
        self.step_count += 1
        o = self.opt
        lr = lr_at(self.step_count - 1, self.sched)
        e = _ext.ext() if self.device.type == "cuda" else None
        p2p = self.backend == "p2p"
        if p2p:
            self._barrier(CH_PARAM)  # nobody reads parameters while they are rewritten
        for bi, b in enumerate(self.buckets):
            so, n = self.shard_off[bi], b["shard"]
            g = self.grad[b["s0"]:b["s0"] + n]
            dec = max(0, min(n, b["start"] + b["decay_n"] - b["s0"]))
            if p2p and self.state.step_range_p2p(so, n, g, self.param_ptrs, b["s0"], dec, lr, o, self.step_count, sqnorm, grad_scale):
                continue  # one kernel: AdamW on this shard and the bf16 store into every rank's parameters
            out = None if p2p else self.bf16[b["s0"]:b["s0"] + n]
            m = self.state.step_range(so, n, g, out, dec, lr, o, self.step_count, sqnorm, grad_scale, need_master=p2p)
            if p2p:  # the updated shard goes straight into every rank's parameters over NVLink
                e.p2p_broadcast_shard(self.param_ptrs, m, b["s0"], n, self.world)
        if p2p:
            self._barrier(CH_PARAM)
        else:
            for b in self.buckets:
                full = self.bf16[b["start"]:b["start"] + b["size"]]
                mine = full[self.rank * b["shard"]:(self.rank + 1) * b["shard"]].clone()
                if dist.get_backend(self.group) == "nccl":
                    dist.all_gather_into_tensor(full, mine, group=self.group)
                else:
                    parts = [torch.empty_like(mine) for _ in range(self.world)]
                    dist.all_gather(parts, mine, group=self.group)
                    full.copy_(torch.cat(parts))
        return sqnorm.sqrt() * grad_scale

    # -------------------------------------------------------------- state (this rank's shards)
    def state_dict(self) -> dict:
        """Sharded state: keys carry the DP rank so every rank saves its own slices."""
        r = self.rank
        st = self.state
        return {f"master.dp{r}": st.master_full(), f"exp_avg.dp{r}": st.m_full(), f"exp_avg_sq.dp{r}": st.v_full(),
                "step": self.step_count}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        r = self.rank
        self.state.load(sd[f"master.dp{r}"], sd[f"exp_avg.dp{r}"], sd[f"exp_avg_sq.dp{r}"])
        self.step_count = int(sd.get("step", self.step_count))

    def check(self) -> None:
        if self.backend == "p2p" and int(self.status.item()):
            raise RuntimeError("distributed optimizer: a peer did not reach a gradient/parameter barrier in time")


class _Null:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *a: Any) -> None:
        return None


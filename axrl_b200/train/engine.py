"""Trainer engine: logprob recompute and the GRPO/PPO/SFT train step on packed micro-batches.

Reference counterpart: ``MegatronWorker`` (``axrl/worker/megatron_worker.py:173-1480``):
``forward_backward_batch`` (:986-1031), the per-token loss rescale (:1041-1057),
``train_step`` (:1059-1123: grad norm, clip, optimizer step) and
``_compute_logprobs_from_local_batches`` (:1195-1303).

Loss scaling follows Megatron's ``calculate_per_token_loss`` contract: each
micro-batch contributes ``loss_mb * denom_mb`` and the accumulated gradient is
divided once by the global ``sum(denom)`` (all micro-batches, all DP ranks).
Here that division is folded into the fused Adam kernel (``grad_scale``).
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

from axrl_b200.configs import MegatronWorkerConfig
from axrl_b200.data.sample import SampleBatch
from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
from axrl_b200.ops import _ext
from axrl_b200.train.optimizer import FlatAdamW
from axrl_b200.train.packing import PackedMicroBatch, pack_rows, split_balanced
from axrl_b200.utils import iostats


@dataclass
class ParallelCtx:
    """Process groups of one trainer rank (None = not parallel along that axis)."""

    dp_group: object | None = None
    tp_group: object | None = None
    dp_size: int = 1
    dp_rank: int = 0
    tp_size: int = 1
    tp_rank: int = 0
    tp_backend: str = "torch"  # "torch" (NCCL/gloo collectives) | "p2p" (NVLink kernels)
    ep_group: object | None = None
    ep_size: int = 1
    ep_backend: str = "torch"
    etp_group: object | None = None  # expert tensor parallelism (ranks holding the same experts' column shards)
    etp_size: int = 1
    pp_group: object | None = None
    pp_size: int = 1
    vpp_size: int = 1  # virtual (interleaved) pipeline stages per rank
    cp_group: object | None = None
    cp_size: int = 1
    zero_backend: str = "p2p"  # distributed optimizer over DP: "p2p" (NVLink) | "nccl" | "off" (replicated)


class TrainEngine:
    def __init__(self, cfg: MegatronWorkerConfig, model_cfg: Qwen3Config, device: torch.device | str = "cpu",
                 dtype: torch.dtype | None = None, par: ParallelCtx | None = None, model: Qwen3Model | None = None):
        self.cfg = cfg
        self.mcfg = model_cfg
        self.device = torch.device(device)
        self.par = par or ParallelCtx()
        dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        from axrl_b200.parallel.tensor_parallel import TPContext

        self.tp = TPContext.from_group(self.par.tp_group, backend=self.par.tp_backend) if self.par.tp_size > 1 else TPContext()
        from axrl_b200.parallel.expert import EPContext

        self.ep = (EPContext.from_group(self.par.ep_group, backend=self.par.ep_backend, hidden=model_cfg.hidden_size,
                                        num_experts=model_cfg.num_experts,
                                        max_rows=(cfg.max_tokens_per_micro_batch + 1024) * max(1, model_cfg.num_experts_per_tok),
                                        etp_group=self.par.etp_group)
                   if self.par.ep_size > 1 or self.par.etp_size > 1 else EPContext())
        from axrl_b200.parallel.context_parallel import CPContext
        from axrl_b200.parallel.pipeline import PPContext

        self.pp = PPContext.from_group(self.par.pp_group, vpp=self.par.vpp_size) if self.par.pp_size > 1 else PPContext()
        self.cp = CPContext.from_group(self.par.cp_group) if self.par.cp_size > 1 else CPContext()
        if model is None and self.pp.enabled and self.pp.vpp > 1:
            from axrl_b200.models.qwen3 import VirtualPipelineModel

            model = VirtualPipelineModel(model_cfg, self.pp, tp=self.tp, ep=self.ep if self.ep.active else None,
                                         cp=self.cp if self.cp.enabled else None)
            model.init_weights(cfg.seed)
            model = model.to(device=self.device, dtype=dtype)
            model.inv_freq = model.chunks[0].inv_freq.float()
        if model is None:
            model = Qwen3Model(model_cfg, tp=self.tp, ep=self.ep if self.ep.active else None,
                               pp=self.pp if self.pp.enabled else None, cp=self.cp if self.cp.enabled else None)
            model.init_weights(cfg.seed)
            model = model.to(device=self.device, dtype=dtype)
            model.inv_freq = model.inv_freq.float()
        self.model = model
        self.role = cfg.model_role
        if self.role == "value":
            # PPO critic: the decoder stack with a scalar value head instead of the LM head
            # (reference axrl/utils/megatron/value_head.py).  The LM head is not trained.
            if self.tp.enabled or self.pp.enabled or self.cp.enabled:
                raise ValueError("the value model runs with tp_size = pp_size = cp_size = 1")
            from axrl_b200.trainer.value_trainer import ValueHead

            self.model.value_head = ValueHead(model_cfg.hidden_size).to(device=self.device, dtype=dtype)
            if getattr(self.model, "lm_head", None) is not None:
                self.model.lm_head.requires_grad_(False)
        from axrl_b200.models.qwen3 import RecomputePolicy

        self.model.set_policy(RecomputePolicy.from_worker_config(cfg))
        if self.device.type == "cuda":
            # deterministic attention backward: dQ without atomics, fixed summation order
            _ext.ext().set_attn_deterministic(bool(cfg.deterministic_mode))
        self.optim = None
        if not cfg.inference_only:
            dp_dist = (cfg.optimizer.use_distributed_optimizer and self.par.dp_group is not None and self.par.dp_size > 1
                       and not self.ep.active and not self.tp.enabled and not self.cp.enabled and self.par.zero_backend != "off")
            if dp_dist:
                from axrl_b200.parallel.zero import BucketedZeroAdamW

                backend = self.par.zero_backend if self.device.type == "cuda" else "nccl"
                self.optim = BucketedZeroAdamW(self.model, cfg.optimizer, cfg.lr_scheduler, group=self.par.dp_group, backend=backend)
            else:
                self.optim = FlatAdamW(self.model, cfg.optimizer, cfg.lr_scheduler)
        self.max_tokens = cfg.max_tokens_per_micro_batch
        self.last_timing: dict[str, float] = {}
        self.release_grads_after_step = False

    # ------------------------------------------------------------------ micro-batches
    def micro_batches(self, batch: SampleBatch) -> list[PackedMicroBatch]:
        lengths = []
        infos = batch.objects.get("merge_info") or [None] * len(batch)
        for r in range(len(batch)):
            lengths.append(infos[r].total_padded if infos[r] is not None else int(batch["seq_len"][r]))
        min_count = 1
        if self.par.dp_group is not None and self.par.dp_size > 1:
            # every DP rank must run the same number of micro-batches
            n = torch.tensor([len(split_balanced(lengths, self.max_tokens))], dtype=torch.int64, device=self.device)  # NCCL: on the GPU
            dist.all_reduce(n, op=dist.ReduceOp.MAX, group=self.par.dp_group)
            min_count = int(n)
        parts = split_balanced(lengths, self.max_tokens * self.cp.size, min_count=min_count)
        if self.cp.enabled:
            from axrl_b200.parallel.context_parallel import pack_rows_cp

            return [pack_rows_cp(batch, p, self.cp) for p in parts if p]
        pad_to = self.tp.size * (16 if self.device.type == "cuda" else 1)
        return [pack_rows(batch, p, pad_to=pad_to) for p in parts if p]

    # ------------------------------------------------------------------ forward
    def _hidden(self, mb: PackedMicroBatch, moe_ctx=None) -> torch.Tensor:  # noqa: ANN001
        return self.model(mb.ids, mb.pos, mb.spec, moe_ctx)

    @torch.no_grad()
    def compute_logprobs(self, batch: SampleBatch, temperature: float = 1.0) -> torch.Tensor:
        """Per-token log p(label) in the batch's (B, S) layout (0 where label is ignored)."""
        self.model.eval()
        B, S = batch["input_ids"].shape
        out = torch.zeros((B, S), dtype=torch.float32)
        if self.pp.enabled:
            return self._compute_logprobs_pp(batch, temperature, out)
        for mb in self.micro_batches(batch):
            dmb = mb.to(self.device)
            h = self._hidden(dmb)
            lp, _ = self.model.logprobs(h, dmb.labels.clamp(min=-1), temperature)
            lp = torch.where(dmb.labels >= 0, lp, torch.zeros_like(lp))
            dense = dmb.unpack(lp.float(), S).cpu()
            if self.device.type == "cuda":
                iostats.add_d2h(dense)
            for li, r in enumerate(mb.rows):
                out[r] += dense[li]
        if self.cp.enabled:  # every position is held by exactly one CP rank
            t = out.to(self.device)
            dist.all_reduce(t, group=self.cp.group)
            out = t.cpu()
        return out

    @torch.no_grad()
    def compute_values(self, batch: SampleBatch) -> torch.Tensor:
        """Value-role engine: V(state) at every label position in the batch's (B, S) layout (0 where
        the label is ignored), the critic predictions PPO's GAE bootstraps from."""
        assert self.role == "value", "compute_values needs model_role='value'"
        self.model.eval()
        B, S = batch["input_ids"].shape
        out = torch.zeros((B, S), dtype=torch.float32)
        for mb in self.micro_batches(batch):
            dmb = mb.to(self.device)
            v = self.model.value_head(self._hidden(dmb))
            v = torch.where(dmb.labels >= 0, v, torch.zeros_like(v))
            dense = dmb.unpack(v.float(), S).cpu()
            for li, r in enumerate(mb.rows):
                out[r] += dense[li]
        return out

    def _act_shape(self, mb: PackedMicroBatch) -> tuple:
        return (mb.num_tokens // self.tp.size, self.mcfg.hidden_size)

    def _act_dtype(self) -> torch.dtype:
        return next(self.model.parameters()).dtype

    def _compute_logprobs_pp(self, batch: SampleBatch, temperature: float, out: torch.Tensor) -> torch.Tensor:
        from axrl_b200.parallel.pipeline import run_forward_only

        S = out.shape[1]
        mbs = self.micro_batches(batch)
        dmbs = [mb.to(self.device) for mb in mbs]

        def fwd(i: int, inp):  # noqa: ANN001, ANN202
            d = dmbs[i]
            return self.model(d.ids, d.pos, d.spec, None, hidden=inp)

        def consume(i: int, h: torch.Tensor) -> None:
            d = dmbs[i]
            lp, _ = self.model.logprobs(h, d.labels.clamp(min=-1), temperature)
            lp = torch.where(d.labels >= 0, lp, torch.zeros_like(lp))
            dense = d.unpack(lp.float(), S).cpu()
            for li, r in enumerate(mbs[i].rows):
                out[r] = dense[li]

        if self.pp.vpp > 1:
            from axrl_b200.parallel.pipeline import run_interleaved_1f1b

            run_interleaved_1f1b(self.pp, self.pp.vpp, len(mbs), lambda i: self._act_shape(mbs[i]), self._act_dtype(), self.device,
                                 lambda i, c, inp: self.model(dmbs[i].ids, dmbs[i].pos, dmbs[i].spec, None, hidden=inp, chunk=c),
                                 consume=consume)
        else:
            run_forward_only(self.pp, len(mbs), lambda i: self._act_shape(mbs[i]), self._act_dtype(), self.device, fwd, consume)
        # the last stage holds the result: broadcast it to every stage
        t = out.to(self.device)
        dist.broadcast(t, src=self.pp.ranks[-1], group=self.pp.group)
        return t.cpu()

    # ------------------------------------------------------------------ train
    def _global_denominator(self, batch: SampleBatch, trainer) -> float:  # noqa: ANN001
        lm = batch["loss_mask"].bool()
        turn_index = batch.get("turn_index", None)
        from axrl_b200.trainer.grpo_trainer import get_num_turns

        nt = get_num_turns(turn_index, lm) if (turn_index is not None and getattr(trainer.config, "micro_batch_denominator_type", "") == "seq_turn") else 0
        d = torch.tensor([float(trainer.compute_micro_batch_denominator(lm, nt))], dtype=torch.float64, device=self.device)
        if self.par.dp_group is not None and self.par.dp_size > 1:
            dist.all_reduce(d, group=self.par.dp_group)
        return float(d)

    def train_step(self, batch: SampleBatch, trainer, temperature: float = 1.0, metrics_every_micro_batch: bool = True) -> dict:  # noqa: ANN001
        """One optimizer step over ``batch`` (this rank's DP slice of one global batch)."""
        assert self.optim is not None, "inference_only engine cannot train"
        t0 = time.perf_counter()
        self.model.train()
        self.optim.zero_grad()
        for m in self.model.modules():  # attention outputs kept for recompute: none may survive a step
            if hasattr(m, "stash"):
                m.stash.clear()
        total_denom = max(self._global_denominator(batch, trainer), 1.0)
        need_entropy = bool(getattr(trainer.config, "entropy_control", None) and
                            (trainer.config.entropy_control.alpha > 0 or trainer.config.entropy_control.compute_entropy))
        S = batch["input_ids"].shape[1]
        mbs = self.micro_batches(batch)
        metrics_acc: list[dict] = []
        if self.pp.enabled:
            metrics_acc = self._forward_backward_pp(batch, mbs, trainer, temperature, need_entropy, metrics_every_micro_batch)
        for i, mb in enumerate(mbs if not self.pp.enabled else []):
            dmb = mb.to(self.device)
            h = self._hidden(dmb)
            if self.role == "value":  # clipped value loss on the critic's predictions
                v = self.model.value_head(h)
                sub = batch.select_rows(mb.rows).to(self.device)
                want = metrics_every_micro_batch or i == len(mbs) - 1
                loss, denom, m = trainer.loss_func({"values": dmb.unpack(v, S)}, sub, with_metrics=want)
                if i == len(mbs) - 1 and hasattr(self.optim, "arm"):
                    self.optim.arm()
                (loss * denom.to(loss.dtype)).backward()
                if want:
                    metrics_acc.append(m)
                continue
            ec = getattr(trainer.config, "entropy_control", None)
            lp, ent = self.model.logprobs(h, dmb.labels.clamp(min=-1), temperature, entropy=need_entropy,
                                          entropy_top_k=max(0, ec.top_k) if ec is not None else 0)
            lp = torch.where(dmb.labels >= 0, lp, torch.zeros_like(lp))
            sub = batch.select_rows(mb.rows).to(self.device)
            if self.device.type == "cuda":
                iostats.add_h2d(*sub.tensors.values())
            if self.cp.enabled:  # this rank trains on the tokens it holds
                from axrl_b200.parallel.context_parallel import local_token_mask

                sub["loss_mask"] = (sub["loss_mask"].bool() & local_token_mask(dmb, S)).to(sub["loss_mask"].dtype)
            outputs = {"log_prob": dmb.unpack(lp, S),
                       "entropy": dmb.unpack(ent, S) if ent is not None else torch.zeros((len(mb.rows), S), device=self.device)}
            if getattr(trainer.config, "compute_accuracy", False) and not self.tp.enabled:
                outputs["argmax"] = dmb.unpack(self.model.argmax_tokens(h.detach()).float(), S).long()
            want = metrics_every_micro_batch or i == len(mbs) - 1
            loss, denom, m = trainer.loss_func(outputs, sub, with_metrics=want)
            if i == len(mbs) - 1 and hasattr(self.optim, "arm"):
                self.optim.arm()  # gradients become final during this backward: reduce buckets as they complete
            (loss * denom.to(loss.dtype)).backward()
            if want:
                metrics_acc.append(m)
        self.optim.fold_param_grads()
        if self.cp.enabled:  # each CP rank back-propagated its own tokens: sum
            dist.all_reduce(self.optim.grad, group=self.cp.group)
        if hasattr(self.optim, "finish_grad_sync"):  # distributed optimizer: reduce-scatter already (mostly) done
            self.optim.finish_grad_sync()
        elif self.par.dp_group is not None and self.par.dp_size > 1:
            if self.ep.active:  # expert weights differ per EP / ETP rank: reduce only the dense gradients
                from axrl_b200.parallel.expert import dense_grad_allreduce

                dense_grad_allreduce(self.model, self.par.dp_group)
            else:
                dist.all_reduce(self.optim.grad, group=self.par.dp_group)  # replicated-optimizer baseline path
        sq = self.optim.grad_sqnorm()
        if self.ep.active:
            from axrl_b200.parallel.expert import expert_params

            sq_e = sum(p.main_grad.float().pow(2).sum() for p in expert_params(self.model)).reshape(1)
            sq_all = sq_e.clone()
            if self.ep.enabled:
                dist.all_reduce(sq_all, group=self.ep.group)
            if self.ep.etp_size > 1:  # and over the column shards
                dist.all_reduce(sq_all, group=self.ep.etp_group)
            sq = (sq - sq_e + sq_all).float()
        if self.tp.enabled:
            from axrl_b200.parallel import tensor_parallel as tpl

            tpl.allreduce_replicated_grads(self.model, self.tp)
            sq = self.optim.grad_sqnorm()
            rep = tpl.replicated_sqnorm(self.model)
            if rep is not None:  # replicated tensors are counted once over the TP group
                sq = sq - rep * (1.0 - 1.0 / self.tp.size)
            sq = sq.reshape(1).float().clone()
            self.tp.comm.all_reduce(sq)
        if self.pp.enabled:  # every stage holds different parameters
            sq = sq.reshape(1).float().clone()
            dist.all_reduce(sq, group=self.pp.group)
        norm = self.optim.step(grad_scale=1.0 / total_denom, sqnorm=sq)
        norm = float(norm)
        for comm in (self.tp.comm, self.ep.comm):
            if comm is not None and hasattr(comm, "check"):
                comm.check()
        if self.release_grads_after_step:
            self.optim.release_grads()
        out = {k: sum(d[k] for d in metrics_acc if k in d) / max(1, sum(1 for d in metrics_acc if k in d))
               for k in {k for d in metrics_acc for k in d}}
        out["grad_norm"] = float(norm)
        out["num_micro_batches"] = len(mbs)
        out["step_time_sec"] = time.perf_counter() - t0
        out["lr"] = self.current_lr()
        if self.device.type == "cuda":
            from axrl_b200.ops import _ext

            _ext.check_kernel_waits()
        from axrl_b200.utils import consistency

        if consistency.enabled() and self.par.dp_group is not None and self.par.dp_size > 1:
            # data-parallel replicas must hold bit-identical parameters after the update
            consistency.check_replicated(((n, p) for n, p in self.model.named_parameters() if not getattr(p, "expert_parallel", False)),
                                         self.par.dp_group)
        return out

    def _forward_backward_pp(self, batch: SampleBatch, mbs: list[PackedMicroBatch], trainer, temperature: float,  # noqa: ANN001
                             need_entropy: bool, every: bool) -> list[dict]:
        from axrl_b200.parallel.pipeline import run_1f1b

        S = batch["input_ids"].shape[1]
        dmbs = [mb.to(self.device) for mb in mbs]
        metrics_acc: list[dict] = []

        def fwd(i: int, inp):  # noqa: ANN001, ANN202
            d = dmbs[i]
            return self.model(d.ids, d.pos, d.spec, None, hidden=inp)

        def loss(i: int, h: torch.Tensor) -> torch.Tensor:
            d = dmbs[i]
            lp, ent = self.model.logprobs(h, d.labels.clamp(min=-1), temperature, entropy=need_entropy)
            lp = torch.where(d.labels >= 0, lp, torch.zeros_like(lp))
            sub = batch.select_rows(mbs[i].rows).to(self.device)
            outputs = {"log_prob": d.unpack(lp, S),
                       "entropy": d.unpack(ent, S) if ent is not None else torch.zeros((len(mbs[i].rows), S), device=self.device)}
            want = every or i == len(mbs) - 1
            l, denom, m = trainer.loss_func(outputs, sub, with_metrics=want)
            if want:
                metrics_acc.append(m)
            return l * denom.to(l.dtype)

        if self.pp.vpp > 1:
            from axrl_b200.parallel.pipeline import run_interleaved_1f1b

            run_interleaved_1f1b(self.pp, self.pp.vpp, len(mbs), lambda i: self._act_shape(mbs[i]), self._act_dtype(), self.device,
                                 lambda i, c, inp: self.model(dmbs[i].ids, dmbs[i].pos, dmbs[i].spec, None, hidden=inp, chunk=c),
                                 loss=loss)
        else:
            run_1f1b(self.pp, len(mbs), lambda i: self._act_shape(mbs[i]), self._act_dtype(), self.device, fwd, loss)
        # metrics live on the last stage
        obj = [metrics_acc if self.pp.is_last else None]
        dist.broadcast_object_list(obj, src=self.pp.ranks[-1], group=self.pp.group)
        return obj[0]

    def current_lr(self) -> float:
        from axrl_b200.train.optimizer import lr_at

        return lr_at(max(0, self.optim.step_count - 1), self.cfg.lr_scheduler) if self.optim else 0.0

    # ------------------------------------------------------------------ weights
    @torch.no_grad()
    def snapshot_weights(self) -> torch.Tensor:
        """CPU copy of all parameters (flat), e.g. the reference-policy snapshot."""
        return self.optim.bf16.detach().to("cpu", copy=True) if self.optim else torch.cat([p.detach().reshape(-1).cpu() for p in self.model.parameters()])

    @torch.no_grad()
    def load_weights(self, flat: torch.Tensor) -> None:
        if self.optim is not None:
            self.optim.bf16.copy_(flat.to(self.optim.bf16.device, non_blocking=True))
        else:
            off = 0
            for p in self.model.parameters():
                p.copy_(flat[off:off + p.numel()].view(p.shape))
                off += p.numel()

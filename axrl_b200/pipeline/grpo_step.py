"""One synthetic GRPO step end to end: rollout -> rewards -> advantages -> packing ->
ref/old logprobs -> train -> weight sync.

This is the driver used by the plumbing run (tiny model on CPU, fp32) and by
the B200 benchmark (Qwen3-8B shape, bf16).  It follows the reference online
loop (``axrl/pipeline/controller.py:1617-1653``, rollout/train/sync of
§3.1-3.4 in the reference docs): prompts are random token ids, the reward is
1 when the response contains ``reward_token``, response lengths are either
sampled freely (stop on EOS / max_new_tokens) or forced through EOS to a
log-normal draw.

Partial rollout (``partial_rollout=True``, the reference's streaming mode with carried-over
trajectories, ``axrl/pipeline/controller.py`` partial rollout): a pool of ``inflight_prompts``
groups stays in generation; a step ends its rollout phase as soon as ``num_prompts`` groups are
complete, aborts the rest (they keep their partial responses) and trains on the completed groups.
The aborted trajectories resume in the next step by re-prefilling prompt + partial response under
the new weights, so the long tail of the response-length distribution never stalls a step.

Colocated single-process mode: the rollout engine reads the trainer's bf16
parameters directly (zero-copy weight sync — the "sync" is the version bump
plus a prefix-cache flush).  ``separate_rollout_copy=True`` keeps an engine-
owned copy and syncs by copying every tensor (what the tiny plumbing config
asks for).
"""

from __future__ import annotations

import copy
import dataclasses
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
from axrl_b200.data.prefix_tree import merge_trajectory_samples
from axrl_b200.data.sample import Sample, SampleBatch
from axrl_b200.models.qwen3 import Qwen3Config
from axrl_b200.pipeline.rewards import group_advantages
from axrl_b200.rollout.engine import GenRequest, GenResult, RolloutEngine
from axrl_b200.train.engine import TrainEngine
from axrl_b200.trainer.grpo_trainer import GrpoTrainer
from axrl_b200.utils import iostats
from axrl_b200.utils.nvtx import nvtx_range


@dataclass
class SyntheticGRPOConfig:
    num_prompts: int = 8
    prompt_len: int = 32
    group_size: int = 4
    max_new_tokens: int = 64
    temperature: float = 1.0
    reward_token: int = 7
    # forced response lengths: log-normal(median, sigma) clipped to [min, max]; None = free sampling
    forced_len_median: float | None = None
    forced_len_sigma: float = 1.0
    forced_len_min: int = 16
    forced_len_max: int = 8192
    eos_token_id: int = 0
    merge_group_prompts: bool = True  # prefix-tree pack each group's shared prompt
    compute_ref_logprobs: bool = True
    # keep the reference-policy weights in device memory (a device-to-device copy before the ref
    # log-prob pass) instead of pinned host memory (a host-to-device copy of the whole model)
    ref_on_device: bool = False
    # partial rollout under data parallelism: stop when the ranks' completed groups add up to the
    # global batch (the groups land where they finish), not when every rank has its own share
    global_stop: bool = True
    compute_old_logprobs: bool = True
    separate_rollout_copy: bool = False
    seed: int = 0
    kv_tokens: int | None = None
    max_batch: int | None = None
    use_cuda_graph: bool = True
    kv_gb: float | None = None  # cap on the KV pool size
    kv_memory_saver: bool = True  # release the KV pool while training (same address on resume)
    partial_rollout: bool = False  # keep unfinished groups in flight across steps
    inflight_prompts: int | None = None  # groups in flight with partial rollout (default 2 x num_prompts)
    extra: dict = field(default_factory=dict)


@dataclass
class _Traj:
    req: GenRequest  # the original request of this trajectory
    out_ids: list[int] = field(default_factory=list)
    out_lps: list[float] = field(default_factory=list)
    done: bool = False
    segments: int = 0  # rollout phases this trajectory took part in


@dataclass
class _Group:
    members: list[_Traj]

    @property
    def done(self) -> bool:
        return all(m.done for m in self.members)


class SyntheticGRPO:
    def __init__(self, model_cfg: Qwen3Config, worker_cfg: MegatronWorkerConfig, grpo_cfg: GrpoTrainerConfig,
                 sc: SyntheticGRPOConfig, device: str | torch.device = "cpu", train_engine: TrainEngine | None = None) -> None:
        self.sc = sc
        self.mcfg = model_cfg
        self.device = torch.device(device)
        self.train = train_engine or TrainEngine(worker_cfg, model_cfg, self.device)
        self.trainer = GrpoTrainer(grpo_cfg)
        self.rng = np.random.default_rng(sc.seed)
        self.ref_weights = None
        if sc.compute_ref_logprobs:
            if sc.ref_on_device and self.device.type == "cuda" and self.train.optim is not None:
                self.ref_weights = self.train.optim.bf16.detach().clone()
            else:
                self.ref_weights = self.train.snapshot_weights()
                if self.device.type == "cuda":
                    self.ref_weights = self.ref_weights.pin_memory()
        rollout_model = self.train.model
        if sc.separate_rollout_copy:
            rollout_model = copy.deepcopy(self.train.model)
            for p in rollout_model.parameters():
                p.requires_grad_(False)
        self.pool: list[_Group] = []  # partial rollout: groups in flight
        self._next_prompt = 0
        inflight = (sc.inflight_prompts or 2 * sc.num_prompts) if sc.partial_rollout else sc.num_prompts
        n_seq = inflight * sc.group_size
        max_ctx = sc.prompt_len + (sc.forced_len_max if sc.forced_len_median else sc.max_new_tokens) + 8
        kv_tokens = sc.kv_tokens or n_seq * (-(-max_ctx // 64) * 64)
        cuda = self.device.type == "cuda"
        if sc.kv_gb is not None:
            per_tok = 2 * model_cfg.num_hidden_layers * model_cfg.num_key_value_heads * model_cfg.head_dim * 2
            kv_tokens = min(kv_tokens, int(sc.kv_gb * (1 << 30)) // per_tok)
        # tensor parallelism: the rollout engine runs on the trainer's own shards (same TP layout) and
        # needs the whole embedding table, gathered from the vocabulary shards after every update
        tp = self.train.tp
        self.embed_full = None
        if tp.enabled:
            emb = self.train.model.embed_tokens
            self.embed_full = torch.empty(emb.shape[0] * tp.size, emb.shape[1], dtype=emb.dtype, device=emb.device)
            self._gather_embedding()
        self.rollout = RolloutEngine(rollout_model, max_batch=sc.max_batch or n_seq, kv_tokens=kv_tokens, page_size=64,
                                     max_context=max_ctx, max_prefill_tokens=max(16384, sc.prompt_len), seed=sc.seed,
                                     use_cuda_graph=sc.use_cuda_graph, eos_token_id=sc.eos_token_id,
                                     kv_memory_saver=cuda and sc.kv_memory_saver,
                                     dp_attention=_ep_active(rollout_model),
                                     tp_group=self.train.par.tp_group if tp.enabled else None, embed_full=self.embed_full)
        if cuda and self.train.optim is not None:
            self.train.release_grads_after_step = True  # the grad buffer is not needed during rollout
        self.weight_version = 0
        self.step_idx = 0
        self.last: dict = {}

    # ------------------------------------------------------------------ pieces
    def _group_requests(self, p: int, tag: str) -> list[GenRequest]:
        sc, V = self.sc, self.mcfg.vocab_size
        prompt = self.rng.integers(1, V, size=sc.prompt_len).tolist()
        reqs = []
        for g in range(sc.group_size):
            forced = None
            if sc.forced_len_median:
                forced = int(np.clip(np.exp(np.log(sc.forced_len_median) + sc.forced_len_sigma * self.rng.standard_normal()),
                                     sc.forced_len_min, sc.forced_len_max))
            reqs.append(GenRequest(rid=f"{tag}-p{p}-g{g}", prompt=prompt, max_new_tokens=forced or sc.max_new_tokens,
                                   temperature=sc.temperature, stop_token_ids=() if forced else (sc.eos_token_id,), forced_len=forced,
                                   forced_token=sc.eos_token_id, seed_stream=self.step_idx * 1_000_000 + p * 1000 + g))
        return reqs

    def make_requests(self) -> list[GenRequest]:
        return [r for p in range(self.sc.num_prompts) for r in self._group_requests(p, f"s{self.step_idx}")]

    def build_samples(self, reqs, results) -> tuple[list[Sample], dict]:  # noqa: ANN001
        sc = self.sc
        samples, scores = [], []
        for r, res in zip(reqs, results):
            scores.append(1.0 if sc.reward_token in res.output_ids else 0.0)
        out: list[Sample] = []
        for p in range(len(reqs) // sc.group_size):
            grp = slice(p * sc.group_size, (p + 1) * sc.group_size)
            adv, mean, std = group_advantages(scores[grp])
            group_samples = []
            for i, (r, res) in enumerate(zip(reqs[grp], results[grp])):
                s = Sample.from_tokens(r.prompt, res.output_ids, reward=scores[grp][i], advantage=float(adv[i]),
                                       rollout_logprobs=res.output_logprobs, trajectory_id=p)
                s.reward_baseline = mean
                group_samples.append(s)
            if sc.merge_group_prompts and sc.group_size > 1:
                m = merge_trajectory_samples(group_samples, align_size=1 if self.device.type == "cpu" else 8)
                m.trajectory_id = p
                out.append(m)
            else:
                out.extend(group_samples)
        resp_tokens = sum(len(res.output_ids) for res in results)
        return out, {"reward_mean": float(np.mean(scores)), "response_tokens": resp_tokens,
                     "mean_response_len": resp_tokens / max(1, len(results))}

    # ------------------------------------------------------------------ the step
    def run_step(self) -> dict:
        sc = self.sc
        t = {}
        io0 = iostats.snapshot()
        t0 = time.perf_counter()
        with nvtx_range("rollout"):
            if sc.partial_rollout:
                reqs, results, pinfo = self._rollout_partial()
            else:
                reqs = self.make_requests()
                self.rollout.acquire_kv()
                results = self.rollout.generate(reqs)
                self.rollout.release_kv()
                pinfo = {}
        t["rollout_s"] = time.perf_counter() - t0

        t1 = time.perf_counter()
        samples, info = self.build_samples(reqs, results)
        batch = SampleBatch.from_samples(samples)
        t["pack_s"] = time.perf_counter() - t1

        t2 = time.perf_counter()
        streamed = (sc.compute_ref_logprobs and sc.compute_old_logprobs and self.device.type == "cuda" and self.train.optim is not None
                    and not self.ref_weights.is_cuda)
        if streamed:
            # reference weights in host memory: copy them in on a side stream while the old-policy
            # pass runs (the KV pool is released in this phase), then swap them in on the device
            cs = getattr(self, "_ref_stream", None) or torch.cuda.Stream(device=self.device)
            self._ref_stream = cs
            ref_dev = torch.empty_like(self.train.optim.bf16)
            cs.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(cs):
                ref_dev.copy_(self.ref_weights, non_blocking=True)
            batch["old_logprobs"] = self.train.compute_logprobs(batch, sc.temperature)
            cur = self.train.optim.bf16.clone()
            torch.cuda.current_stream().wait_stream(cs)
            ref_dev.record_stream(torch.cuda.current_stream())
            self.train.load_weights(ref_dev)
            del ref_dev
            batch["ref_logprobs"] = self.train.compute_logprobs(batch, sc.temperature)
            self.train.load_weights(cur)
            del cur
        elif sc.compute_ref_logprobs:
            cur = self.train.snapshot_weights() if self.device.type == "cpu" else None
            if cur is None:
                cur = self.train.optim.bf16.clone() if self.train.optim else None
            self.train.load_weights(self.ref_weights)
            batch["ref_logprobs"] = self.train.compute_logprobs(batch, sc.temperature)
            self.train.load_weights(cur)
            del cur
        if sc.compute_old_logprobs and not streamed:
            batch["old_logprobs"] = self.train.compute_logprobs(batch, sc.temperature)
        else:
            batch["old_logprobs"] = batch["rollout_logprobs"].clone()
        if "ref_logprobs" not in batch.tensors:
            batch["ref_logprobs"] = batch["old_logprobs"]
        t["logprob_s"] = time.perf_counter() - t2

        t3 = time.perf_counter()
        with nvtx_range("train_step"):
            metrics = self.train.train_step(batch, self.trainer, temperature=sc.temperature)
        t["train_s"] = time.perf_counter() - t3

        t4 = time.perf_counter()
        self.sync_weights()
        t["sync_s"] = time.perf_counter() - t4
        self.step_idx += 1
        io1 = iostats.snapshot()
        t["h2d_bytes"], t["d2h_bytes"] = io1[0] - io0[0], io1[1] - io0[1]
        trained_tokens = int(batch["seq_len"].sum())
        out = {**metrics, **info, **pinfo, **t, "trained_tokens": trained_tokens, "num_samples": len(samples),
               "sequences": len(results), "total_tokens": sum(len(r.prompt) + len(x.output_ids) for r, x in zip(reqs, results))}
        self.last = out
        return out

    def _rollout_partial(self) -> tuple[list[GenRequest], list[GenResult], dict]:
        """Streaming rollout phase: top the pool up, generate until ``num_prompts`` groups are
        complete, abort the rest (partial responses kept) and return the completed groups."""
        sc = self.sc
        inflight = sc.inflight_prompts or 2 * sc.num_prompts
        while len(self.pool) < inflight:
            self.pool.append(_Group([_Traj(r) for r in self._group_requests(self._next_prompt, "q")]))
            self._next_prompt += 1
        live: dict[str, _Traj] = {}
        reqs = []
        resumed = 0
        for g in self.pool:
            for m in g.members:
                if m.done:
                    continue
                r, n = m.req, len(m.out_ids)
                rid = f"{r.rid}@{self.step_idx}"
                resumed += n > 0
                reqs.append(dataclasses.replace(r, rid=rid, prompt=list(r.prompt) + m.out_ids, max_new_tokens=max(1, r.max_new_tokens - n),
                                                forced_len=None if r.forced_len is None else r.forced_len - n, gen_prefix=tuple(m.out_ids)))
                live[rid] = m

        def absorb(res: GenResult) -> None:
            m = live.pop(res.rid)
            m.out_ids += res.output_ids
            m.out_lps += res.output_logprobs
            m.segments += 1
            if res.finish_reason != "abort":
                m.done = True

        self.rollout.acquire_kv()
        self.rollout.add_requests(reqs)
        par = self.train.par
        if sc.global_stop and par.dp_group is not None and par.dp_size > 1:
            # data-parallel ranks stop together, once the ranks' completed groups add up to the
            # global batch (num_prompts per rank): one all-reduce per decode burst, so no rank idles
            # in the next collective while another finishes its longest group
            import torch.distributed as dist

            mine = torch.zeros(2, dtype=torch.int64, device=self.device)
            every = torch.zeros(2 * par.dp_size, dtype=torch.int64, device=self.device)
            while True:
                if self.rollout.waiting or self.rollout.running:
                    for res in self.rollout.step():
                        absorb(res)
                mine[0] = sum(g.done for g in self.pool)
                mine[1] = int(bool(self.rollout.waiting or self.rollout.running))
                dist.all_gather_into_tensor(every, mine, group=par.dp_group)
                done, busy = every.view(-1, 2)[:, 0].tolist(), every.view(-1, 2)[:, 1].tolist()
                # every rank needs at least one group of its own to train on
                if (sum(done) >= sc.num_prompts * par.dp_size and min(done) >= 1) or sum(busy) == 0:
                    break
            take_n = len(self.pool)  # every group this rank completed
        else:
            while sum(g.done for g in self.pool) < sc.num_prompts and (self.rollout.waiting or self.rollout.running):
                for res in self.rollout.step():
                    absorb(res)
            take_n = sc.num_prompts
        aborted = 0
        for res in self.rollout.abort_all():
            aborted += 1
            absorb(res)
        self.rollout.release_kv()
        take = [g for g in self.pool if g.done][:take_n]
        self.pool = [g for g in self.pool if not any(g is t for t in take)]
        out_reqs, out_res = [], []
        for g in take:
            for m in g.members:
                out_reqs.append(m.req)
                out_res.append(GenResult(m.req.rid, m.out_ids, m.out_lps, "stop", len(m.req.prompt)))
        info = {"groups_done": len(take), "resumed_trajectories": resumed, "aborted_trajectories": aborted,
                "carried_groups": len(self.pool), "multi_segment_trajectories": sum(m.segments > 1 for g in take for m in g.members)}
        return out_reqs, out_res, info

    @torch.no_grad()
    def _gather_embedding(self) -> None:
        """The whole embedding table from the TP ranks' vocabulary shards, into the same buffer (the
        rollout engine's CUDA graphs hold its address)."""
        import torch.distributed as dist

        dist.all_gather_into_tensor(self.embed_full, self.train.model.embed_tokens.detach().contiguous(), group=self.train.par.tp_group)

    def sync_weights(self) -> None:
        """Trainer -> rollout weight sync (in-process)."""
        if self.sc.separate_rollout_copy:
            self.rollout.update_weights_from_model(self.train.model)
        if self.embed_full is not None:
            self._gather_embedding()
        self.rollout.reset_prefix_cache()
        self.weight_version += 1


def _ep_active(model) -> bool:  # noqa: ANN001
    """An expert-parallel model: every rank runs its own requests and the engines step in lockstep
    (data-parallel attention), since each MoE layer's dispatch is collective over the EP group."""
    ep = getattr(model, "ep", None)
    return bool(ep is not None and getattr(ep, "active", False))

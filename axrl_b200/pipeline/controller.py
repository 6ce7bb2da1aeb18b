"""Pipeline controller: the online RL loop and the other run modes.

Reference: ``PipelineController`` (``axrl/pipeline/controller.py:74-1795``):

* ``online_rl_train`` (:1617-1653): schedule GRPO groups (more than one sync window needs),
  stream results, normalise group rewards, drop zero-std groups, pack trajectories, train on
  ``model_sync_every_n_global_updates`` global batches, sync weights, checkpoint, eval — while
  unfinished groups keep generating across the sync (partial rollout, :846-865, :1101-1176);
* ``eval_only``, ``sft_train``, ``replay_rl_train`` and ``mismatch_test`` (:1456-1779).

Deployment here is one process per GPU: the rollout engine and the trainer share the GPU
(colocated) and the bf16 weights; rollout actors are coroutines; queues are asyncio.  The stage
manager pauses generation around training (aborted requests resume from their partial output
after the sync) and releases/re-acquires the trainer's gradient buffer around rollout.
"""

from __future__ import annotations

import asyncio
import json
import logging
import time
from collections import defaultdict
from pathlib import Path
from typing import Any

import numpy as np
import torch

from axrl_b200.data.sample import SampleBatch
from axrl_b200.metrics.response_metric import aggregate_response_metrics
from axrl_b200.pipeline.config import PipelineExperimentConfig
from axrl_b200.pipeline.rewards import group_advantages
from axrl_b200.pipeline.rollout_actor import RolloutActor, RolloutRuntime
from axrl_b200.runtime.task_queue import AsyncTaskQueue

logger = logging.getLogger(__name__)

RESULT_TIMEOUT_S = 30.0


class PipelineController:
    def __init__(self, config: PipelineExperimentConfig, recipe: Any, *, device: str | torch.device | None = None,
                 model_cfg: Any = None) -> None:
        self.config = config
        self.recipe = recipe
        self.device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
        self.model_cfg = model_cfg
        self.global_step = 0
        self.metrics_log: list[dict] = []
        self.train_dataset = None
        self.pending: dict[str, list] = defaultdict(list)
        self.group_sizes: dict[str, int] = {}
        self.output_dir = Path(config.mismatch_test.output_dir).parent / config.controller.output_dir_name

    # ------------------------------------------------------------------ init
    async def initialize(self) -> None:
        from axrl_b200.models.qwen3 import resolve_preset
        from axrl_b200.rollout.engine import RolloutEngine
        from axrl_b200.train.engine import TrainEngine
        from axrl_b200.trainer.grpo_trainer import GrpoTrainer
        from axrl_b200.worker.infer_router import InferenceRouter
        from axrl_b200.worker.rollout_worker import RolloutWorker

        c = self.config
        await self.recipe.register_datasets()
        self.check_configs()
        mcfg = self.model_cfg or resolve_preset(c.megatron_worker.model.name)
        self.train = TrainEngine(c.megatron_worker, mcfg, self.device)
        self.trainer = GrpoTrainer(c.grpo)
        rw = c.rollout_worker
        max_ctx = c.train_sampling_config.max_total_tokens
        kv_tokens = int(rw.max_running_requests * (max_ctx + 128))
        self.engine = RolloutEngine(self.train.model, max_batch=rw.max_running_requests, kv_tokens=kv_tokens, page_size=rw.kv_page_size,
                                    max_context=max_ctx, use_cuda_graph=rw.use_cuda_graph, seed=c.megatron_worker.seed)
        self.worker = RolloutWorker(self.engine, c.train_sampling_config, continue_after_abort=rw.continue_generation_after_abort)
        self.router = InferenceRouter([self.worker], max_imbalance=rw.max_imbalance)
        self.rollout_queue: AsyncTaskQueue = AsyncTaskQueue(max_running=c.controller.max_running_requests, name="rollout")
        self.result_queue: AsyncTaskQueue = AsyncTaskQueue(name="result")
        self.services = await self.recipe.start_services()
        runtime = RolloutRuntime(rollout_worker=self.router, local_processors=dict(self.recipe.initialize_local_processors("actor-0")),
                                 shared_workers=self.recipe.initialize_shared_workers(self.services), config=c)
        self.actors = [RolloutActor(self.recipe, runtime, self.rollout_queue, self.result_queue, num_loops=max(1, c.controller.max_running_requests))]
        for a in self.actors:
            a.start()

    def check_configs(self) -> None:
        o = self.config.online_rl_train
        if o.strict_on_policy:
            assert o.model_sync_every_n_global_updates == 1 and o.batch_rollout_for_n_global_updates == 1, \
                "strict_on_policy requires syncing and rolling out every global update"
        assert o.batch_rollout_for_n_global_updates >= o.model_sync_every_n_global_updates, \
            "batch_rollout_for_n_global_updates must cover at least one sync window"
        if o.checkpoint_every_n_global_updates:
            assert o.checkpoint_every_n_global_updates % o.model_sync_every_n_global_updates == 0, \
                "checkpoint cadence must be a multiple of the model-sync cadence"

    # ------------------------------------------------------------------ entry
    async def start(self) -> dict:
        await self.initialize()
        try:
            mode = self.config.controller.run_mode
            if mode == "online_rl_train":
                return await self.run_online_rl_train()
            if mode == "eval_only":
                return await self.run_evals()
            raise NotImplementedError(f"run mode {mode} is driven by axrl_b200.pipeline.modes")
        finally:
            await self.shutdown()

    async def shutdown(self) -> None:
        for a in getattr(self, "actors", []):
            await a.stop()
        if getattr(self, "worker", None) is not None:
            self.worker.shutdown()
        if getattr(self, "services", None) is not None:
            await self.recipe.stop_services(self.services)
        await self.recipe.shutdown()

    # ------------------------------------------------------------------ scheduling
    def groups_per_sync(self) -> int:
        c = self.config
        G = c.online_rl_train.num_rollouts_per_conversation
        total = c.megatron_worker.global_batch_size * c.online_rl_train.model_sync_every_n_global_updates
        assert total % G == 0, "global_batch_size * model_sync_every_n_global_updates must be divisible by the group size"
        return total // G

    async def schedule_groups(self, conversations: list) -> None:
        G = self.config.online_rl_train.num_rollouts_per_conversation
        items = []
        for conv in conversations:
            gid = conv.conversation_id + f"@{self.global_step}:{len(self.group_sizes)}"
            self.group_sizes[gid] = G
            for g in range(G):
                c = conv.deep_copy()
                c.extra["group_id"] = gid
                c.extra["group_index"] = g
                items.append(c)
        await self.rollout_queue.put_many(items)

    def normalize_group_rewards(self, group: list) -> None:
        scores = [r.metric.score for r in group]
        adv, mean, std = group_advantages(scores)
        if self.train_dataset is not None:
            self.train_dataset.update_score_history(group[0].conversation.conversation_id, scores)
        for r, a in zip(group, adv):
            r.metric.score_mean, r.metric.score_std = mean, std
            r.reward, r.reward_baseline, r.scalar_advantage = r.metric.score, mean, float(a)
            if r.trace is not None:
                for s in r.trace.turn_samples:
                    s.reward, s.reward_baseline = r.metric.score, mean
                    s.advantage = np.where(s.loss_mask, np.float32(a), np.float32(0.0)).astype(np.float32)

    async def stream_groups(self, target_valid: int) -> tuple[list[list], list]:
        """Collect results until ``target_valid`` complete groups pass the zero-std filter."""
        valid, dropped = [], []
        o = self.config.online_rl_train
        while len(valid) < target_valid:
            r = await self.result_queue.get(timeout=RESULT_TIMEOUT_S)
            if r is None:
                for a in self.actors:
                    a.check_health()
                logger.info("waiting for rollouts: %s", self.rollout_queue.get_stats())
                continue
            await self.result_queue.complete()
            gid = r.conversation.extra["group_id"]
            self.pending[gid].append(r)
            if len(self.pending[gid]) < self.group_sizes[gid]:
                continue
            group = self.pending.pop(gid)
            self.normalize_group_rewards(group)
            if o.filter_zero_std and np.std([g.metric.score for g in group]) < 1e-8:
                dropped.append(group)
                continue
            valid.append(group)
        return valid, dropped

    # ------------------------------------------------------------------ train
    def pack_groups(self, groups: list[list]) -> SampleBatch:
        from axrl_b200.data.rollout_trace import pack_rollout_traces_for_train_batches

        traces = []
        for group in groups:
            for r in group:
                r.trace.trajectory_id = len(traces)
                traces.append(r.trace)
        c = self.config
        samples = pack_rollout_traces_for_train_batches(traces, c.megatron_worker.model.seq_length,
                                                         allow_prefix_sharing=c.controller.allow_prefix_merging)
        total = sum(int(s.loss_mask.sum()) for s in samples)
        expect = sum(int(t.turn_samples[i].loss_mask.sum()) for t in traces for i in range(len(t.turn_samples)))
        assert total <= expect, "packing must not create trainable tokens"
        return SampleBatch.from_samples(samples)

    def train_on(self, batch: SampleBatch) -> list[dict]:
        from axrl_b200.data.global_batch_iterator import build_global_batches_for_dp_rank

        c = self.config
        G = c.online_rl_train.num_rollouts_per_conversation
        gbs_traj = max(1, c.megatron_worker.global_batch_size)
        out = []
        batches = build_global_batches_for_dp_rank(batch, global_batch_size=gbs_traj, dp_size=1, dp_rank=0,
                                                   padding_sample_length=c.megatron_worker.padding_sample_length)
        for b in batches:
            b["old_logprobs"] = self.train.compute_logprobs(b, c.train_sampling_config.temperature)
            if "ref_logprobs" not in b.tensors:
                b["ref_logprobs"] = b["old_logprobs"]
            m = self.train.train_step(b, self.trainer, temperature=c.train_sampling_config.temperature)
            self.global_step += 1
            m["global_step"] = self.global_step
            out.append(m)
        _ = G
        return out

    async def run_online_rl_train(self) -> dict:
        c = self.config
        o = c.online_rl_train
        assert self.train_dataset is not None, "recipe must provide a train dataset (controller.train_dataset)"
        per_sync = self.groups_per_sync()
        scheduled = per_sync * o.batch_rollout_for_n_global_updates // o.model_sync_every_n_global_updates
        await self.schedule_groups(self.train_dataset.sample(scheduled, o.sample_type))
        history = []
        while self.global_step < o.max_global_updates:
            t0 = time.time()
            valid, dropped = await self.stream_groups(per_sync)
            t_roll = time.time() - t0
            # keep the pipeline full: top up the groups consumed by this window
            await self.schedule_groups(self.train_dataset.sample(len(valid) + len(dropped), o.sample_type))
            self.worker.pause_generation()  # partial rollout: in-flight requests resume after the sync
            t1 = time.time()
            batch = self.pack_groups(valid)
            step_metrics = self.train_on(batch)
            t_train = time.time() - t1
            t2 = time.time()
            self.engine.reset_prefix_cache()  # colocated: weights are shared, only the cache is stale
            self.worker.resume_generation()
            t_sync = time.time() - t2
            res = [r for g in valid for r in g]
            m = {"timing/rollout_seconds": t_roll, "timing/train_seconds": t_train, "timing/sync_seconds": t_sync,
                 **aggregate_response_metrics([r.metric for r in res], "Valid-Rollouts", t_roll),
                 **{f"train/{k}": v for k, v in step_metrics[-1].items() if isinstance(v, (int, float))},
                 "group_filter_type__zero_std_dropped": float(len(dropped))}
            history.append(m)
            self.metrics_log.append(m)
            logger.info("step %d %s", self.global_step, json.dumps({k: round(v, 4) for k, v in m.items() if isinstance(v, float)}))
        return {"history": history}

    async def run_evals(self) -> dict:
        return {}

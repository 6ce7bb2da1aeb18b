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
from pathlib import Path as _Path
from typing import Any

import numpy as np
import torch

from axrl_b200.data.sample import SampleBatch
from axrl_b200.metrics.response_metric import aggregate_response_metrics, aggregate_response_metrics_by_subset
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
        self.value = self.value_trainer = None
        self.value_step = 0
        if c.value_worker is not None and self.is_ppo_training():
            from axrl_b200.trainer.value_trainer import ValueTrainer

            self.value = TrainEngine(c.value_worker, mcfg, self.device)  # the critic starts from the same architecture
            self.value_trainer = ValueTrainer(c.grpo.ppo_value)
        rw = c.rollout_worker
        max_ctx = c.train_sampling_config.max_total_tokens
        kv_tokens = int(rw.max_running_requests * (max_ctx + 128))
        self.engine = RolloutEngine(self.train.model, max_batch=rw.max_running_requests, kv_tokens=kv_tokens, page_size=rw.kv_page_size,
                                    max_context=max_ctx, use_cuda_graph=rw.use_cuda_graph, seed=c.megatron_worker.seed,
                                    dp_attention=_ep_active(self.train.model))
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
        self.check_ppo_value_configs(self.config)
        o = self.config.online_rl_train
        if o.strict_on_policy:
            assert o.model_sync_every_n_global_updates == 1 and o.batch_rollout_for_n_global_updates == 1, \
                "strict_on_policy requires syncing and rolling out every global update"
        assert o.batch_rollout_for_n_global_updates >= o.model_sync_every_n_global_updates, \
            "batch_rollout_for_n_global_updates must cover at least one sync window"
        if o.checkpoint_every_n_global_updates:
            assert o.checkpoint_every_n_global_updates % o.model_sync_every_n_global_updates == 0, \
                "checkpoint cadence must be a multiple of the model-sync cadence"

    @staticmethod
    def check_ppo_value_configs(c: PipelineExperimentConfig) -> None:
        """PPO needs a critic whose layout matches the actor (reference
        ``axrl/pipeline/controller.py:152-200``)."""
        g, actor, value = c.grpo, c.megatron_worker, c.value_worker

        def need(ok: bool, msg: str) -> None:
            if not ok:
                raise ValueError(msg)

        if g.loss_type == "ppo" or g.ppo_value is not None:
            need(c.controller.run_mode == "online_rl_train", "PPO with a value worker runs in controller.run_mode='online_rl_train' only")
        if g.loss_type == "ppo":
            need(g.ppo_value is not None, "grpo.loss_type='ppo' requires grpo.ppo_value")
            need(value is not None, "grpo.loss_type='ppo' requires value_worker")
            need(value.model_role == "value", "PPO value_worker.model_role must be 'value'")
            need(actor.model_role == "actor", "PPO megatron_worker.model_role must be 'actor'")
            need(value.world_size() == actor.world_size(),
                 f"PPO value_worker world_size ({value.world_size()}) must match the actor's ({actor.world_size()})")
            need(value.model.seq_length == actor.model.seq_length, "PPO value_worker seq_length must match the actor's")
            need(value.checkpoint_dir != actor.checkpoint_dir, "PPO actor and value workers need different checkpoint_dir values")
            need(g.is_base_logprobs == "old_logprobs", "the PPO actor loss uses old_logprobs as the policy-ratio base")
        if g.ppo_value is not None:
            need(g.loss_type == "ppo", "grpo.ppo_value is only supported with grpo.loss_type='ppo'")
            need(value is not None, "grpo.ppo_value requires value_worker")
            need(not g.ppo_value.use_stateless_value_model, "grpo.ppo_value.use_stateless_value_model is not implemented")

    def is_ppo_training(self) -> bool:
        return self.config.grpo.loss_type == "ppo"

    def prepare_ppo_training_samples(self, b: SampleBatch) -> None:
        """Critic predictions before its update (``old_values``), terminal-token rewards, token-level
        GAE -> per-token advantages and returns (reference ``controller.py:1310-1339``)."""
        from axrl_b200.trainer.ppo_utils import build_terminal_token_rewards, compute_gae, normalize_over_valid_tokens_in_batch

        pv = self.config.grpo.ppo_value
        old_values = self.value.compute_values(b).float()
        lm = b["loss_mask"].bool()
        rewards = build_terminal_token_rewards(b["reward"].float(), lm)
        adv, ret = compute_gae(rewards, old_values, lm, gamma=pv.gamma, gae_lambda=pv.gae_lambda)
        if self.config.grpo.normalize_advantages_over_valid_tokens_in_batch:
            adv = normalize_over_valid_tokens_in_batch(adv, lm)
        b["old_values"] = old_values
        b["returns"] = ret
        b["advantage"] = adv.to(b["advantage"].dtype)

    # ------------------------------------------------------------------ entry
    async def start(self) -> dict:
        await self.initialize()
        try:
            mode = self.config.controller.run_mode
            if mode == "online_rl_train":
                return await self.run_online_rl_train()
            if mode == "eval_only":
                return {"results": await self.run_eval_only()}
            if mode == "sft_train":
                return {"curve": await self.run_sft_train()}
            if mode == "replay_rl_train":
                return await self.run_replay_rl_train()
            if mode == "mismatch_test":
                return await self.run_mismatch_test()
            raise ValueError(f"unknown run mode {mode}")
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

    # ------------------------------------------------------------------ checkpoints
    def checkpoint_root(self) -> Path:
        return self.config.megatron_worker.get_checkpoint_dir()

    def save_checkpoint(self) -> Path:
        """torch_dist checkpoint of model + optimizer + controller/dataset state (retries inside),
        plus an HF safetensors export with rotation when ``save_hf_checkpoint``.  Reference:
        ``BaseController.save_checkpoint`` / ``save_hf_checkpoint`` (``axrl/controller/base_controller.py:153-203``)."""
        import shutil

        from axrl_b200.train.checkpoint import save_dist_checkpoint, save_hf_checkpoint

        mw = self.config.megatron_worker
        extra = {"global_step": self.global_step,
                 "dataset_state": self.train_dataset.state_dict() if self.train_dataset is not None else None}
        d = save_dist_checkpoint(self.checkpoint_root(), self.global_step, self.train.model, self.train.optim, extra=extra,
                                 most_recent_k=mw.most_recent_checkpoint_k)
        if mw.save_hf_checkpoint:
            hf_root = self.checkpoint_root().parent / "hf"
            save_hf_checkpoint(self.train.model, hf_root / f"step_{self.global_step:07d}")
            olds = sorted(p for p in hf_root.glob("step_*") if p.is_dir())
            for old in olds[:-mw.most_recent_checkpoint_k]:
                shutil.rmtree(old, ignore_errors=True)
        return d

    def load_checkpoint_if_existed(self) -> bool:
        from axrl_b200.train.checkpoint import latest_iteration, load_dist_checkpoint

        root = self.checkpoint_root()
        if latest_iteration(root) is None:
            return False
        common = load_dist_checkpoint(root, self.train.model, self.train.optim)
        extra = common.get("extra", {})
        self.global_step = int(extra.get("global_step", common.get("iteration", 0)))
        if self.train_dataset is not None and extra.get("dataset_state"):
            self.train_dataset.load_state_dict(extra["dataset_state"])
        logger.info("resumed from %s at global_step=%d", root, self.global_step)
        return True

    def save_checkpoint_if_needed(self) -> None:
        n = self.config.online_rl_train.checkpoint_every_n_global_updates
        if n and self.global_step % n == 0:
            self.save_checkpoint()

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
            m: dict = {}
            if self.is_ppo_training():
                t0 = time.time()
                self.prepare_ppo_training_samples(b)
                vm = self.value.train_step(b, self.value_trainer)
                self.value_step += 1
                m.update({f"value/{k}": v for k, v in vm.items() if isinstance(v, (int, float))})
                m["timing/value_train_seconds"] = time.time() - t0
                if self.value_step <= c.grpo.ppo_value.num_value_only_updates:
                    m["actor_trained"] = 0.0  # value-only warmup: the critic learns before the actor moves
                    out.append(m)
                    continue
            m.update(self.train.train_step(b, self.trainer, temperature=c.train_sampling_config.temperature))
            self.global_step += 1
            m["global_step"] = self.global_step
            out.append(m)
        _ = G
        return out

    async def run_online_rl_train(self) -> dict:
        c = self.config
        o = c.online_rl_train
        assert self.train_dataset is not None, "recipe must provide a train dataset (controller.train_dataset)"
        self.load_checkpoint_if_existed()
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
            self.save_checkpoint_if_needed()
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

    # ------------------------------------------------------------------ other run modes
    def get_test_datasets(self) -> list[tuple[str, Any]]:
        """(name, dataset) pairs: the controller's ``test_datasets`` or the recipe's."""
        ds = getattr(self, "test_datasets", None)
        if ds is None and hasattr(self.recipe, "get_test_datasets"):
            ds = self.recipe.get_test_datasets()
        return list(ds or [])

    async def collect_results(self, n: int) -> list:
        out = []
        while len(out) < n:
            r = await self.result_queue.get(timeout=RESULT_TIMEOUT_S)
            if r is None:
                for a in self.actors:
                    a.check_health()
                continue
            await self.result_queue.complete()
            out.append(r)
        return out

    async def run_eval_rollouts(self) -> list:
        """Roll out every test conversation once (``smoke_eval_rollouts`` caps the total); metrics per
        dataset under ``eval_<name>/``; rollouts saved when ``save_eval_rollouts``."""
        from axrl_b200.utils.zst_utils import save_zst

        all_results = []
        budget = self.config.controller.smoke_eval_rollouts
        for name, ds in self.get_test_datasets():
            if budget is not None and budget <= 0:
                break
            convs = [c.deep_copy() for c in ds.conversations]
            if budget is not None:
                convs = convs[:budget]
                budget -= len(convs)
            for i, c in enumerate(convs):
                c.extra["group_id"] = f"eval:{name}:{c.conversation_id}@{self.global_step}"
                c.extra["group_index"] = i
            t0 = time.time()
            await self.rollout_queue.put_many(convs)
            results = await self.collect_results(len(convs))
            dt = time.time() - t0
            m = aggregate_response_metrics([r.metric for r in results], f"eval_{name}", dt)
            m[f"eval_{name}/eval_time_sec"] = dt
            subset_key = getattr(getattr(ds, "config", None), "subset_key", None) or getattr(ds, "subset_key", None)
            if subset_key:  # per-subset breakdown, e.g. by source benchmark
                m.update(aggregate_response_metrics_by_subset(results, subset_key, f"eval_{name}"))
            self.metrics_log.append(m)
            if self.config.controller.save_eval_rollouts:
                save_zst(results, self.output_dir / f"eval_rollouts-{name}-step{self.global_step}.zst")
            all_results.extend(results)
        return all_results

    async def run_evals(self) -> list:
        if not self.get_test_datasets():
            logger.info("no test datasets configured; skipping evaluation")
            return []
        return await self.run_eval_rollouts()

    async def run_eval_only(self) -> list:
        results = await self.run_eval_rollouts()
        assert results, "eval_only needs at least one test dataset with conversations"
        return results

    def build_sft_samples(self, dataset: Any) -> SampleBatch:
        samples = self.recipe.build_sft_samples(dataset)
        batch = SampleBatch.from_samples(samples)
        batch["trajectory_id"] = torch.arange(len(batch), dtype=torch.long)
        return batch

    async def run_sft_train(self) -> list[dict]:
        """Supervised fine-tuning over the recipe's SFT samples for ``megatron_worker.num_epochs``
        epochs; the eval loss is the token-mean NLL of the test datasets."""
        from axrl_b200.configs import SftTrainerConfig
        from axrl_b200.data.global_batch_iterator import build_global_batches_for_dp_rank
        from axrl_b200.trainer.sft_trainer import SftTrainer

        c = self.config
        train = self.build_sft_samples(self.train_dataset)
        evals = [self.build_sft_samples(ds) for _, ds in self.get_test_datasets()]
        trainer = SftTrainer(getattr(c, "sft", None) or SftTrainerConfig())
        curve = []
        for epoch in range(c.megatron_worker.num_epochs):
            t0 = time.time()
            g = torch.Generator().manual_seed(self.global_step)
            order = torch.randperm(len(train), generator=g).tolist()
            shuffled = train.select_rows(order)
            last = {}
            for b in build_global_batches_for_dp_rank(shuffled, global_batch_size=c.megatron_worker.global_batch_size, dp_size=1,
                                                      dp_rank=0, padding_sample_length=c.megatron_worker.padding_sample_length):
                last = self.train.train_step(b, trainer)
                self.global_step += 1
            row = {"global_step": float(self.global_step), "epoch": float(epoch), "train_loss": float(last.get("loss", float("nan"))),
                   "train_grad_norm": float(last.get("grad_norm", float("nan"))), "timing/train_seconds": time.time() - t0}
            if evals:
                tot, cnt = 0.0, 0.0
                for eb in evals:
                    lp = self.train.compute_logprobs(eb)
                    m = eb["loss_mask"].bool()
                    tot += float(-lp[m].sum())
                    cnt += float(m.sum())
                row["eval_loss"] = tot / max(cnt, 1.0)
            curve.append(row)
            self.metrics_log.append(row)
        return curve

    def select_replay_groups(self, groups: list[list]) -> list[list]:
        """Re-normalise each loaded group and drop zero-std groups (as the online loop does)."""
        keep = []
        for g in groups:
            self.normalize_group_rewards(g)
            if self.config.online_rl_train.filter_zero_std and np.std([r.metric.score for r in g]) < 1e-8:
                continue
            keep.append(g)
        return keep

    async def run_replay_rl_train(self) -> dict:
        """Train on recorded data: a saved sample set, or saved rollout groups re-packed here."""
        from pathlib import Path as _P

        from axrl_b200.utils.zst_utils import load_zst

        rc = self.config.replay_rl_train
        assert (rc.sample_dict_path is None) != (rc.rollout_groups_path is None), \
            "replay_rl_train requires exactly one of sample_dict_path or rollout_groups_path"
        if rc.sample_dict_path is not None:
            batch = load_zst(_P(rc.sample_dict_path))
        else:
            groups = self.select_replay_groups(load_zst(_P(rc.rollout_groups_path)))
            batch = self.pack_groups(groups)
        if not self.config.controller.allow_prefix_merging and "merge_info" in batch.objects:
            batch.objects.pop("merge_info")
        t0 = time.time()
        metrics = self.train_on(batch)
        out = {"train_metrics": metrics, "timing/train_seconds": time.time() - t0}
        self.metrics_log.append({k: v for k, v in out.items() if isinstance(v, float)})
        return out

    async def run_mismatch_test(self) -> dict:
        """Roll out one global batch (zero-std filter off, or load saved rollouts), recompute the
        trainer's log-probs of every sampled token, save the samples and report the rollout-vs-trainer
        mismatch (optionally against a baseline run)."""
        from datetime import datetime, timezone

        from axrl_b200.metrics.report_mismatch import MCoreRunMetrics, MismatchReportTask, MismatchRunResult, report_mismatch
        from axrl_b200.utils.zst_utils import load_zst, save_zst

        mc = self.config.mismatch_test
        name = mc.name
        for d in (mc.get_output_dir(), mc.get_result_dir(), mc.get_log_dir(), mc.get_fig_dir()):
            d.mkdir(parents=True, exist_ok=True)
        stem = mc._sanitize_name(name)
        result_path = mc.get_result_dir() / f"result-{stem}.zst"
        save_zst(MismatchRunResult(success=False, grpo_config=self.config.grpo.model_copy()), result_path)
        rollout_path = mc.get_result_dir() / "data" / f"valid_rollouts-{stem}.zst"
        samples_path = mc.get_result_dir() / "data" / f"samples-{stem}.zst"
        t0 = time.time()
        if rollout_path.exists() and not mc.override_rollouts_if_exists:
            groups = load_zst(rollout_path)
        else:
            keep = self.config.online_rl_train.filter_zero_std
            self.config.online_rl_train.filter_zero_std = False
            try:
                n = self.groups_per_sync()
                await self.schedule_groups(self.train_dataset.sample(n, self.config.online_rl_train.sample_type))
                groups, _ = await self.stream_groups(n)
            finally:
                self.config.online_rl_train.filter_zero_std = keep
            save_zst(groups, rollout_path)
        t_roll = time.time() - t0
        metrics_r = [r.metric for g in groups for r in g]
        resp = aggregate_response_metrics(metrics_r, "Mismatch-Rollout", None)
        tokens = sum(m.response_length for m in metrics_r)
        self.worker.pause_generation()
        batch = self.pack_groups(groups)
        t1 = time.time()
        batch["old_logprobs"] = self.train.compute_logprobs(batch, self.config.train_sampling_config.temperature)
        batch["ref_logprobs"] = batch["old_logprobs"].clone()  # no update happened: the reference policy is the current one
        t_mcore = time.time() - t1
        save_zst(batch, samples_path)
        base = None
        if mc.baseline_samples_path is not None:
            base = mc.baseline_samples_path
        elif mc.baseline_name is not None:
            base = str(mc.get_result_dir() / "data" / f"samples-{mc._sanitize_name(mc.baseline_name)}.zst")
        if base is not None and not _Path(base).exists():
            raise FileNotFoundError(f"baseline sample set not found at {base}")
        ts = datetime.now(tz=timezone.utc).strftime("%Y%m%d-%H%M%S")
        mm = report_mismatch(MismatchReportTask(exp_name=name, exp_sample_data_path=str(samples_path), baseline_sample_data_path=base,
                                                baseline_name=mc.baseline_name or "baseline",
                                                output_fig_path=str(mc.get_fig_dir() / f"mismatch_report-{stem}-{ts}.svg"),
                                                output_txt_path=str(mc.get_log_dir() / f"top_mismatch-{stem}-{ts}.log")))
        result = MismatchRunResult(success=True, grpo_config=self.config.grpo.model_copy(),
                                   metadata={"pipeline_config": self.config.model_dump(mode="json")}, response_metrics=resp,
                                   rollout_throughput=tokens / t_roll if t_roll > 0 else None,
                                   mcore=MCoreRunMetrics(end_to_end_time_sec=t_mcore), mismatch_metrics=mm)
        save_zst(result, result_path)
        return {"result_path": str(result_path), "mismatch": mm}


def _ep_active(model) -> bool:  # noqa: ANN001
    """An expert-parallel model: every rank runs its own requests and the engines step in lockstep
    (data-parallel attention), since each MoE layer's dispatch is collective over the EP group."""
    ep = getattr(model, "ep", None)
    return bool(ep is not None and getattr(ep, "active", False))

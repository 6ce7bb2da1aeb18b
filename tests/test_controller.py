"""Controller on CPU with the tiny model: streaming groups through rollout actors, group
normalisation, packing, training, partial-rollout pause/resume; plus queue and router logic."""

import asyncio

import pytest
import torch

from axrl_b200.runtime.task_queue import AsyncTaskQueue
from axrl_b200.worker.infer_router import InferenceRouter


def test_task_queue_limits_and_timeout():
    async def go():
        q = AsyncTaskQueue(max_running=2)
        await q.put_many([1, 2, 3])
        a, b = await q.get(), await q.get()
        assert (a, b) == (1, 2)
        assert await q.get(timeout=0.05) is None  # running limit reached
        await q.complete()
        assert await q.get(timeout=0.5) == 3
        assert q.get_stats()["timeouts"] == 1

    asyncio.run(go())


def test_router_affinity_and_imbalance():
    r = InferenceRouter([object(), object()], max_imbalance=1)
    assert r.assign("s1") == 0
    r.load[0] = 5
    assert r.assign("s2") == 1  # least loaded
    assert r.assign("s1") == 1  # affinity broken: imbalance 5 > 1


def test_online_rl_loop_tiny_cpu():
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.config import PipelineExperimentConfig
    from axrl_b200.pipeline.controller import PipelineController
    from axrl_b200.recipe.synthetic_recipe import SyntheticTokenRecipe

    torch.manual_seed(0)
    c = PipelineExperimentConfig()
    c.megatron_worker.global_batch_size = 8  # trajectories per global batch
    c.megatron_worker.model.seq_length = 256
    c.online_rl_train.num_rollouts_per_conversation = 4
    c.online_rl_train.model_sync_every_n_global_updates = 1
    c.online_rl_train.batch_rollout_for_n_global_updates = 2
    c.online_rl_train.max_global_updates = 2
    c.online_rl_train.checkpoint_every_n_global_updates = None
    c.train_sampling_config.max_new_tokens = 24
    c.train_sampling_config.max_total_tokens = 96
    c.rollout_worker.max_running_requests = 16
    c.controller.max_running_requests = 16
    c.grpo.loss_type = "grpo"
    recipe = SyntheticTokenRecipe(c, num_prompts=8, prompt_len=16)
    ctl = PipelineController(c, recipe, device="cpu", model_cfg=resolve_preset("tiny"))
    ctl.train_dataset = recipe.dataset
    out = asyncio.run(ctl.start())
    hist = out["history"]
    assert len(hist) == 2 and ctl.global_step == 2
    assert all(h["Valid-Rollouts/num"] == 8 for h in hist)
    assert all(torch.isfinite(torch.tensor(h["train/grad_norm"])) for h in hist)

"""Controller on CPU with the tiny model: streaming groups through rollout actors, group
normalisation, packing, training, partial-rollout pause/resume; plus queue and router logic."""

import asyncio
from unittest import mock

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


def _ctl(tmp_path, mode):
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.config import PipelineExperimentConfig
    from axrl_b200.pipeline.controller import PipelineController
    from axrl_b200.recipe.synthetic_recipe import SyntheticTokenRecipe

    torch.manual_seed(0)
    c = PipelineExperimentConfig()
    c.controller.run_mode = mode
    c.megatron_worker.global_batch_size = 8
    c.megatron_worker.model.seq_length = 256
    c.megatron_worker.num_epochs = 3
    c.online_rl_train.num_rollouts_per_conversation = 4
    c.online_rl_train.model_sync_every_n_global_updates = 1
    c.online_rl_train.batch_rollout_for_n_global_updates = 1
    c.train_sampling_config.max_new_tokens = 16
    c.train_sampling_config.max_total_tokens = 64
    c.rollout_worker.max_running_requests = 16
    c.controller.max_running_requests = 16
    c.mismatch_test.output_dir = str(tmp_path / "mm")
    recipe = SyntheticTokenRecipe(c, num_prompts=8, prompt_len=16)
    ctl = PipelineController(c, recipe, device="cpu", model_cfg=resolve_preset("tiny"))
    ctl.output_dir = tmp_path / "out"
    ctl.train_dataset = recipe.dataset
    return ctl


def test_eval_only_and_sft_modes(tmp_path):
    ctl = _ctl(tmp_path, "eval_only")
    out = asyncio.run(ctl.start())
    assert len(out["results"]) == 4 and any("eval_synthetic_test/num" in m for m in ctl.metrics_log)
    assert list((tmp_path / "out").glob("eval_rollouts-*.zst"))
    ctl = _ctl(tmp_path, "sft_train")
    curve = asyncio.run(ctl.start())["curve"]
    assert len(curve) == 3 and curve[-1]["train_loss"] < curve[0]["train_loss"] and "eval_loss" in curve[0]


def test_mismatch_then_replay(tmp_path):
    from axrl_b200.utils.zst_utils import load_zst

    ctl = _ctl(tmp_path, "mismatch_test")
    out = asyncio.run(ctl.start())
    mm = out["mismatch"]
    # same fp32 weights, same math: the rollout engine and the trainer agree closely
    assert mm["mismatch/cur-exp/num_tokens"] > 0 and mm["mismatch/cur-exp/abs_diff_mean"] < 1e-3
    res = load_zst(out["result_path"])
    assert res.success and res.mismatch_metrics == mm
    rollouts = list((tmp_path / "mm" / "results" / "data").glob("valid_rollouts-*.zst"))
    assert rollouts and list((tmp_path / "mm" / "results" / "figs").glob("*.svg"))
    ctl = _ctl(tmp_path, "replay_rl_train")
    ctl.config.replay_rl_train.rollout_groups_path = str(rollouts[0])
    ctl.config.online_rl_train.filter_zero_std = False
    out = asyncio.run(ctl.start())
    assert out["train_metrics"] and all(torch.isfinite(torch.tensor(m["grad_norm"])) for m in out["train_metrics"])


def test_checkpoint_save_and_resume(tmp_path):
    ctl = _ctl(tmp_path, "online_rl_train")
    c = ctl.config
    c.megatron_worker.checkpoint_dir = str(tmp_path / "ckpt")
    c.megatron_worker.save_hf_checkpoint = True
    c.megatron_worker.most_recent_checkpoint_k = 1
    c.online_rl_train.max_global_updates = 2
    c.online_rl_train.checkpoint_every_n_global_updates = 1
    asyncio.run(ctl.start())
    assert (tmp_path / "ckpt" / "latest_checkpointed_iteration.txt").read_text() == "2"
    assert len(list((tmp_path / "ckpt").glob("iter_*"))) == 1 and len(list((tmp_path / "hf").glob("step_*"))) == 1
    params = {n: p.detach().clone() for n, p in ctl.train.model.named_parameters()}
    ctl2 = _ctl(tmp_path, "online_rl_train")
    ctl2.config.megatron_worker.checkpoint_dir = str(tmp_path / "ckpt")
    ctl2.config.online_rl_train.max_global_updates = 2  # already reached: resumes and stops
    asyncio.run(ctl2.start())
    assert ctl2.global_step == 2
    for n, p in ctl2.train.model.named_parameters():
        torch.testing.assert_close(p, params[n])


def _ppo_config():
    from axrl_b200.configs import MegatronWorkerConfig, PPOValueConfig
    from axrl_b200.pipeline.config import PipelineExperimentConfig

    c = PipelineExperimentConfig()
    c.megatron_worker.global_batch_size = 8
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
    c.grpo.loss_type = "ppo"
    c.grpo.ppo_value = PPOValueConfig(gamma=1.0, gae_lambda=0.95, num_value_only_updates=1)
    c.value_worker = MegatronWorkerConfig(model_role="value", checkpoint_dir="checkpoints/value", seed=7)
    c.value_worker.model.seq_length = 256
    c.value_worker.lr_scheduler.lr_warmup_steps = 0
    return c


def test_ppo_with_value_worker_tiny_cpu():
    """PPO through the controller: the critic predicts old values, terminal rewards -> GAE give
    per-token advantages and returns, the critic trains with the clipped value loss, and the actor
    waits for the value-only warmup update before it trains."""
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.controller import PipelineController
    from axrl_b200.recipe.synthetic_recipe import SyntheticTokenRecipe

    torch.manual_seed(0)
    c = _ppo_config()
    recipe = SyntheticTokenRecipe(c, num_prompts=8, prompt_len=16)
    ctl = PipelineController(c, recipe, device="cpu", model_cfg=resolve_preset("tiny"))
    ctl.train_dataset = recipe.dataset
    seen = {}
    orig = ctl.prepare_ppo_training_samples

    def spy(b):
        orig(b)
        # the last batch: the critic has been updated, so its values are no longer the zero init
        seen["adv"], seen["ret"], seen["mask"] = b["advantage"].clone(), b["returns"].clone(), b["loss_mask"].bool().clone()

    ctl.prepare_ppo_training_samples = spy
    # a reward that every batch sees both values of (token presence on a random tiny model is
    # usually 0 for a whole batch, which leaves the critic with nothing to fit)
    with mock.patch("axrl_b200.recipe.synthetic_recipe.token_presence_reward", lambda ids, tok: float(bool(ids) and ids[0] % 2 == 0)):
        asyncio.run(ctl.start())
    assert ctl.global_step == 2 and ctl.value_step == 3  # one value-only warmup update, then both train
    m = seen["mask"]
    assert torch.isfinite(seen["adv"]).all() and (seen["adv"][~m] == 0).all()
    # per-token advantages vary along a response (GAE over the critic's values), unlike GRPO's constant
    rows = [r for r in range(m.shape[0]) if m[r].sum() > 2]
    assert any(seen["adv"][r][m[r]].unique().numel() > 1 for r in rows)
    vw = ctl.value.model.value_head.weight
    assert vw.abs().sum() > 0  # the critic's head moved away from its zero init


def test_ppo_config_checks():
    import pytest

    from axrl_b200.pipeline.controller import PipelineController

    c = _ppo_config()
    PipelineController.check_ppo_value_configs(c)
    bad = _ppo_config()
    bad.value_worker.model_role = "actor"
    with pytest.raises(ValueError, match="model_role"):
        PipelineController.check_ppo_value_configs(bad)
    bad = _ppo_config()
    bad.value_worker.checkpoint_dir = bad.megatron_worker.checkpoint_dir
    with pytest.raises(ValueError, match="checkpoint_dir"):
        PipelineController.check_ppo_value_configs(bad)
    bad = _ppo_config()
    bad.grpo.loss_type = "grpo"
    with pytest.raises(ValueError, match="ppo_value"):
        PipelineController.check_ppo_value_configs(bad)

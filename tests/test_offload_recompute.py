"""Recompute policies, activation offload and optimizer-state offload (CPU; the GPU variants run
in test_gpu_engine.py)."""

import pytest
import torch

from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig, MegatronWorkerConfig
from axrl_b200.models.qwen3 import Qwen3Model, RecomputePolicy, resolve_preset
from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens


def _grads(policy: RecomputePolicy, preset: str = "tiny"):
    torch.manual_seed(0)
    m = Qwen3Model(resolve_preset(preset))
    m.init_weights(1)
    m.set_policy(policy)
    T = 40
    ids = torch.randint(1, 1000, (T,))
    pos = torch.cat([torch.arange(25), torch.arange(15)])
    spec = causal_spec_from_cu_seqlens([0, 25, 40])
    h = m(ids, pos, spec)
    (h.float().square().mean()).backward()
    return {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}


@pytest.mark.parametrize("policy", [
    RecomputePolicy("full"),
    RecomputePolicy("full", "uniform", 2),
    RecomputePolicy("full", "block", 1),
    RecomputePolicy("selective", modules=("core_attn", "layernorm", "mlp")),
    RecomputePolicy(offload_layers=1),
    RecomputePolicy(offload_layers=2, offload_double_buffer=True),
])
def test_recompute_and_offload_keep_gradients(policy):
    ref = _grads(RecomputePolicy())
    got = _grads(policy)
    assert ref.keys() == got.keys()
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=1e-6, msg=n)


def test_selective_moe_and_shared_expert_recompute():
    ref = _grads(RecomputePolicy(), "tiny-moe")
    got = _grads(RecomputePolicy("selective", modules=("moe", "layernorm")), "tiny-moe")
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=1e-6, msg=n)


def test_policy_groups_and_validation():
    assert RecomputePolicy("full", "uniform", 3).groups(7) == [(0, 3, True), (3, 6, True), (6, 7, True)]
    assert RecomputePolicy("full", "block", 2).groups(4) == [(0, 1, True), (1, 2, True), (2, 3, False), (3, 4, False)]
    assert RecomputePolicy("selective").groups(2) == [(0, 1, False), (1, 2, False)]
    with pytest.raises(ValueError):
        RecomputePolicy.from_worker_config(MegatronWorkerConfig(recompute_granularity="selective", recompute_modules=["mla_up_proj"]))
    with pytest.raises(ValueError):
        RecomputePolicy.from_worker_config(MegatronWorkerConfig(cpu_offloading=True, cpu_offloading_num_layers=0))
    p = RecomputePolicy.from_worker_config(MegatronWorkerConfig(recompute_granularity="full", recompute_method="uniform",
                                                                recompute_num_layers=4, cpu_offloading=True,
                                                                cpu_offloading_num_layers=2, cpu_offloading_double_buffering=True))
    assert (p.granularity, p.method, p.num_layers, p.offload_layers, p.offload_double_buffer) == ("full", "uniform", 4, 2, True)


def test_unsupported_settings_are_rejected():
    from pydantic import ValidationError

    from axrl_b200.configs import RolloutWorkerConfig

    with pytest.raises(ValidationError):
        MegatronWorkerConfig(fp8="e4m3")
    with pytest.raises(ValidationError):
        RolloutWorkerConfig(kv_cache_dtype="fp8_e4m3")


@pytest.mark.parametrize("fraction", [0.3, 1.0])
def test_optimizer_state_offload_matches_device_state(fraction):
    from axrl_b200.train.optimizer import FlatAdamW

    sched = MCoreLrSchedulerConfig(lr_warmup_steps=0, max_lr=1e-2)
    outs = []
    for frac in (0.0, fraction):
        torch.manual_seed(0)
        m = Qwen3Model(resolve_preset("tiny"))
        m.init_weights(3)
        opt = FlatAdamW(m, MCoreOptimizerConfig(lr=1e-2, optimizer_cpu_offload=frac > 0, optimizer_offload_fraction=frac), sched)
        assert opt.state.offloaded == round(opt.numel * frac)
        for step in range(3):
            opt.zero_grad()
            g = torch.Generator().manual_seed(step)
            opt.grad.copy_(torch.randn(opt.numel, generator=g))
            opt.step()
        outs.append((opt.bf16.clone(), opt.state_dict()))
    (b0, s0), (b1, s1) = outs
    torch.testing.assert_close(b1, b0)
    for k in ("master", "exp_avg", "exp_avg_sq"):
        torch.testing.assert_close(s1[k], s0[k])

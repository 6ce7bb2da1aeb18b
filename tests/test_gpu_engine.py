"""GPU rollout/train engines on a small Qwen3 (head_dim 128): graph decode == eager decode,
forced lengths, rollout logprobs vs trainer recompute, and one GRPO step."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from axrl_b200.models.qwen3 import Qwen3Config

    return Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=128)


def _model(seed=0):
    from axrl_b200.models.qwen3 import Qwen3Model

    m = Qwen3Model(_cfg())
    m.init_weights(seed)
    m = m.to("cuda", torch.bfloat16)
    m.inv_freq = m.inv_freq.float()
    return m


def _reqs(n=6, forced=None):
    from axrl_b200.rollout.engine import GenRequest

    g = torch.Generator().manual_seed(0)
    out = []
    for i in range(n):
        prompt = torch.randint(1, 2048, (40 + 7 * i,), generator=g).tolist()
        out.append(GenRequest(rid=f"r{i}", prompt=prompt, max_new_tokens=50, temperature=1.0, stop_token_ids=(),
                              forced_len=None if forced is None else forced[i], forced_token=3, seed_stream=i))
    return out


def test_graph_decode_matches_eager():
    from axrl_b200.rollout.engine import RolloutEngine

    m = _model()
    a = RolloutEngine(m, max_batch=8, kv_tokens=4096, max_context=256, use_cuda_graph=True, seed=5, burst=8)
    b = RolloutEngine(m, max_batch=8, kv_tokens=4096, max_context=256, use_cuda_graph=False, seed=5, burst=8)
    ra, rb = a.generate(_reqs()), b.generate(_reqs())
    for x, y in zip(ra, rb):
        assert x.output_ids == y.output_ids
        assert len(x.output_ids) == 50
        # same tokens; log-probs agree to bf16 rounding (split-K decode GEMMs add partials in any order)
        torch.testing.assert_close(torch.tensor(x.output_logprobs), torch.tensor(y.output_logprobs), atol=1e-2, rtol=0)
    a.release_graphs()


def test_forced_lengths_and_group_sharing():
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    m = _model()
    eng = RolloutEngine(m, max_batch=16, kv_tokens=8192, max_context=512, seed=1, eos_token_id=3, burst=16)
    prompt = list(range(10, 140))  # 130 tokens: 2 full pages + a partial page copied per member
    reqs = [GenRequest(rid=f"g{i}", prompt=prompt, max_new_tokens=300, forced_len=L, forced_token=3, seed_stream=i)
            for i, L in enumerate([1, 5, 17, 64, 65, 200])]
    res = eng.generate(reqs)
    for r, L in zip(res, [1, 5, 17, 64, 65, 200]):
        assert len(r.output_ids) == L and r.output_ids[-1] == 3 and r.finish_reason == "stop"
    assert len({tuple(r.output_ids[:4]) for r in res if len(r.output_ids) >= 4}) > 1  # members sample independently
    assert eng.bm.num_available() == eng.num_pages - 1  # every page returned (cached ones evictable)
    eng.release_graphs()


def test_rollout_logprobs_match_trainer_recompute():
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.rollout.engine import RolloutEngine
    from axrl_b200.train.engine import TrainEngine

    m = _model(3)
    eng = RolloutEngine(m, max_batch=8, kv_tokens=4096, max_context=256, seed=2)
    reqs = _reqs(4)
    res = eng.generate(reqs)
    samples = [Sample.from_tokens(r.prompt, x.output_ids, rollout_logprobs=x.output_logprobs) for r, x in zip(reqs, res)]
    batch = SampleBatch.from_samples(samples)
    tr = TrainEngine(MegatronWorkerConfig(inference_only=True), _cfg(), "cuda", model=m)
    lp = tr.compute_logprobs(batch)
    mask = batch["loss_mask"]
    diff = (lp - batch["rollout_logprobs"])[mask].abs()
    assert diff.mean().item() < 0.02 and diff.max().item() < 0.5, (diff.mean().item(), diff.max().item())
    eng.release_graphs()


def test_grpo_step_on_gpu_reduces_loss_direction():
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.pipeline.grpo_step import SyntheticGRPO, SyntheticGRPOConfig

    wc = MegatronWorkerConfig(recompute_granularity="full")
    wc.lr_scheduler.lr_warmup_steps = 0
    sc = SyntheticGRPOConfig(num_prompts=4, prompt_len=64, group_size=4, max_new_tokens=48, reward_token=5, merge_group_prompts=True)
    pipe = SyntheticGRPO(_cfg(), wc, GrpoTrainerConfig(loss_type="grpo2"), sc, "cuda")
    m1 = pipe.run_step()
    m2 = pipe.run_step()
    for m in (m1, m2):
        assert m["trained_tokens"] > 0 and torch.isfinite(torch.tensor(m["loss"]))
    pipe.rollout.release_graphs()


def test_vmm_buffer_pause_resume_keeps_address():
    from axrl_b200.runtime.vmm import VmmBuffer

    buf = VmmBuffer((3, 1000, 64), torch.bfloat16, tag="test_vmm")
    ptr = buf.tensor.data_ptr()
    x = torch.randn(3, 1000, 64, device="cuda").bfloat16()
    buf.tensor.copy_(x)
    buf.pause(backup=True)
    buf.resume()
    assert buf.tensor.data_ptr() == ptr
    torch.testing.assert_close(buf.tensor, x, atol=0, rtol=0)
    buf.pause(backup=False)
    buf.resume()
    buf.tensor.fill_(1.0)
    assert buf.tensor.float().sum().item() == 3 * 1000 * 64
    buf.free()


def test_kv_release_acquire_and_preemption():
    """Graph decode across a KV release/acquire cycle, and a KV pool too small for the batch
    (the newest sequences are preempted and resumed by re-prefill)."""
    from axrl_b200.rollout.engine import RolloutEngine

    m = _model(4)
    forced = [120, 7, 200, 64, 150, 90]
    eng = RolloutEngine(m, max_batch=8, kv_tokens=4096, max_context=512, seed=3, burst=8, kv_memory_saver=True)
    r1 = eng.generate(_reqs(6, forced))
    eng.release_kv()
    eng.acquire_kv()
    r2 = eng.generate(_reqs(6, forced))
    for a, b, L in zip(r1, r2, forced):
        assert len(a.output_ids) == len(b.output_ids) == L
    eng.release_graphs()

    # 10 pages of 64 tokens for six sequences that grow to up to 6 pages each
    forced = [300, 7, 280, 64, 250, 90]
    small = RolloutEngine(m, max_batch=8, kv_tokens=640, max_context=512, seed=3, burst=8, eos_token_id=3)
    reqs = _reqs(6, forced)
    for r in reqs:
        r.max_new_tokens = 300
    res = small.generate(reqs)
    assert small.stats.get("preempted", 0) > 0
    for r, L in zip(res, forced):
        assert len(r.output_ids) == len(r.output_logprobs) == L and r.output_ids[-1] == 3 and r.finish_reason == "stop"
    assert [r.rid for r in res] == [q.rid for q in reqs]
    small.release_graphs()


def test_filtered_sampling_in_graph_decode():
    """top-k / penalties / allowed-token sets run inside the captured decode graph."""
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    m = _model(6)
    eng = RolloutEngine(m, max_batch=8, kv_tokens=4096, max_context=256, seed=4, burst=8)
    reqs = [GenRequest(rid="allowed", prompt=list(range(3, 40)), max_new_tokens=24, allowed_token_ids=[100, 101, 102], seed_stream=1),
            GenRequest(rid="norepeat", prompt=list(range(3, 40)), max_new_tokens=30, top_k=1, presence_penalty=1e4, seed_stream=2),
            GenRequest(rid="topp", prompt=list(range(9, 30)), max_new_tokens=16, top_p=0.5, min_p=0.05, seed_stream=3)]
    res = {r.rid: r for r in eng.generate(reqs)}
    assert set(res["allowed"].output_ids) <= {100, 101, 102} and len(res["allowed"].output_ids) == 24
    assert len(set(res["norepeat"].output_ids)) == 30
    assert len(res["topp"].output_ids) == 16 and all(lp <= 0 for lp in res["topp"].output_logprobs)
    assert any(k[1] for k in eng.graphs)  # a filtered-mode graph was captured
    eng.release_graphs()


def test_recompute_reuses_attention_and_matches_plain_backward():
    """Checkpointed layers keep (o, lse) of the first forward for the replay in backward: the
    gradients equal those of the same model trained without recompute, and the attention kernel
    runs once per layer instead of twice."""
    from axrl_b200.ops import core
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    torch.manual_seed(0)
    T = 700
    ids = torch.randint(0, 2048, (T,), device="cuda")
    labels = torch.randint(0, 2048, (T,), device="cuda")
    pos = torch.cat([torch.arange(300), torch.arange(400)]).int().cuda()
    spec = causal_spec_from_cu_seqlens([0, 300, 700]).to("cuda")
    grads = {}
    for recompute in (False, True):
        m = _model(5)
        m.train()
        m.recompute = recompute
        lp, _ = m.logprobs(m(ids, pos, spec), labels)
        lp.float().sum().backward()
        grads[recompute] = {k: p.grad.float().clone() for k, p in m.named_parameters() if p.grad is not None}
        assert all(not layer.self_attn.stash.items for layer in m.layers), "every stashed output consumed"
    for k, g in grads[False].items():
        rel = ((grads[True][k] - g).norm() / (g.norm() + 1e-12)).item()
        assert rel < 1e-2, f"{k}: {rel}"
    assert core.AttnStash.pushing is False


def test_recompute_policies_and_activation_offload_on_gpu():
    """Grouped / block / selective recompute and pinned-host activation offload (with and without
    the side-stream double buffer) give the gradients of plain backward."""
    from axrl_b200.models.qwen3 import RecomputePolicy
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    torch.manual_seed(0)
    T = 512
    ids = torch.randint(0, 2048, (T,), device="cuda")
    labels = torch.randint(0, 2048, (T,), device="cuda")
    pos = torch.cat([torch.arange(200), torch.arange(312)]).int().cuda()
    spec = causal_spec_from_cu_seqlens([0, 200, 512]).to("cuda")
    policies = [RecomputePolicy(), RecomputePolicy("full", "uniform", 2), RecomputePolicy("full", "block", 1),
                RecomputePolicy("selective", modules=("core_attn", "layernorm", "mlp")), RecomputePolicy(offload_layers=2),
                RecomputePolicy(offload_layers=1, offload_double_buffer=True)]
    grads = []
    for pol in policies:
        m = _model(5)
        m.train()
        m.set_policy(pol)
        lp, _ = m.logprobs(m(ids, pos, spec), labels)
        lp.float().sum().backward()
        torch.cuda.synchronize()
        grads.append({k: p.grad.float().clone() for k, p in m.named_parameters() if p.grad is not None})
    for pol, gr in zip(policies[1:], grads[1:]):
        for k, g in grads[0].items():
            rel = ((gr[k] - g).norm() / (g.norm() + 1e-12)).item()
            assert rel < 1e-2, f"{pol}: {k}: {rel}"


def test_optimizer_state_offload_on_gpu_matches_device_state():
    """The tail of the fp32 optimizer state in pinned host memory, updated on the CPU, tracks the
    fused device update (same parameters after three steps, within bf16 rounding)."""
    from axrl_b200.configs import MCoreLrSchedulerConfig, MCoreOptimizerConfig
    from axrl_b200.train.optimizer import FlatAdamW

    sched = MCoreLrSchedulerConfig(lr_warmup_steps=0, max_lr=1e-3)
    outs = []
    for frac in (0.0, 0.4):
        m = _model(7)
        opt = FlatAdamW(m, MCoreOptimizerConfig(lr=1e-3, optimizer_cpu_offload=frac > 0, optimizer_offload_fraction=frac), sched)
        assert opt.state.offloaded == round(opt.numel * frac)
        for step in range(3):
            opt.zero_grad()
            g = torch.Generator(device="cuda").manual_seed(step)
            opt.grad.copy_(torch.randn(opt.numel, device="cuda", generator=g))
            opt.step()
        torch.cuda.synchronize()
        outs.append((opt.bf16.float().clone(), opt.state.master_full().float().cpu()))
    assert (outs[0][0] - outs[1][0]).abs().max().item() <= 2 ** -7 * outs[0][0].abs().max().item()
    torch.testing.assert_close(outs[1][1], outs[0][1], rtol=1e-5, atol=1e-6)


def test_qwen35_style_hybrid_on_gpu_matches_fp32_and_rollout():
    """Gated attention output, zero-centered norms, Gated DeltaNet layers and a shared expert on the GPU
    path (head dim 128, full rotary: the shapes the GPU kernels cover): bf16 trainer log-probs track
    the fp32 CPU model, and rollout log-probs track the trainer's recomputation."""
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens
    from axrl_b200.rollout.engine import RolloutEngine
    from axrl_b200.train.engine import TrainEngine

    cfg = Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=4, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256,
                      shared_expert_intermediate_size=256, layer_types=["linear_attention", "full_attention"] * 2,
                      linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
                      attn_output_gate=True, zero_centered_norm=True)
    cpu = Qwen3Model(cfg)
    cpu.init_weights(4)
    gpu = Qwen3Model(cfg)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.to("cuda", torch.bfloat16)
    gpu.inv_freq = gpu.inv_freq.float()
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(1, 2048, (96,), generator=g)
    pos = torch.cat([torch.arange(40), torch.arange(56)]).int()
    spec = causal_spec_from_cu_seqlens([0, 40, 96])
    labels = torch.roll(ids, -1)
    with torch.no_grad():
        lp_ref = cpu.logprobs(cpu(ids, pos, spec), labels)[0]
        lp = gpu.logprobs(gpu(ids.cuda(), pos.cuda(), spec.to("cuda")), labels.cuda())[0].float().cpu()
    d = (lp - lp_ref).abs()
    assert d.mean().item() < 0.03 and d.max().item() < 0.3, (d.mean().item(), d.max().item())

    for p in gpu.parameters():
        p.requires_grad_(False)
    eng = RolloutEngine(gpu, max_batch=4, kv_tokens=2048, max_context=256, seed=3)
    reqs = _reqs(3)
    res = eng.generate(reqs)
    samples = [Sample.from_tokens(r.prompt, x.output_ids, rollout_logprobs=x.output_logprobs) for r, x in zip(reqs, res)]
    batch = SampleBatch.from_samples(samples)
    tr = TrainEngine(MegatronWorkerConfig(inference_only=True), cfg, "cuda", model=gpu)
    lp2 = tr.compute_logprobs(batch)
    mask = batch["loss_mask"]
    diff = (lp2 - batch["rollout_logprobs"])[mask].abs()
    assert diff.mean().item() < 0.02 and diff.max().item() < 0.5, (diff.mean().item(), diff.max().item())
    eng.release_graphs()

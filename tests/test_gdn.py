"""Hybrid linear / full-attention models (Gated DeltaNet layers, Qwen3-Next / 3.5 style; the
reference trains them through Megatron's ``gated_delta_net`` variant,
``axrl/utils/megatron/magi_forward.py:790-848``): the chunked delta rule against its recurrence,
packed sequences kept independent, a GRPO step, and rollout log-probs (prefill state + per-token
decode) against the trainer's packed forward."""

import torch

from axrl_b200.models.gdn import gated_delta_chunked, gated_delta_chunked_varlen, gated_delta_recurrent


def _cfg():
    from axrl_b200.models.qwen3 import resolve_preset

    return resolve_preset("tiny-gdn")


def test_chunked_delta_rule_matches_recurrence():
    torch.manual_seed(0)
    for L, chunk in [(5, 4), (70, 16), (129, 64)]:
        H, dk, dv = 3, 8, 6
        q = torch.nn.functional.normalize(torch.randn(L, H, dk), dim=-1) / dk ** 0.5
        k = torch.nn.functional.normalize(torch.randn(L, H, dk), dim=-1)
        v, g, beta = torch.randn(L, H, dv), -torch.rand(L, H), torch.rand(L, H)
        S0 = torch.randn(H, dk, dv) * 0.1
        o1, s1 = gated_delta_chunked(q, k, v, g, beta, S0, chunk=chunk)
        o2, s2 = gated_delta_recurrent(q, k, v, g, beta, S0)
        torch.testing.assert_close(o1, o2, atol=1e-5, rtol=1e-4)
        torch.testing.assert_close(s1, s2, atol=1e-5, rtol=1e-4)


def test_varlen_chunked_matches_per_sequence():
    """All packed sequences at once (chunks batched, padded tails) = one sequence at a time, values and
    gradients."""
    torch.manual_seed(1)
    lens, H, dk, dv, C = [5, 16, 70, 33, 1], 2, 8, 4, 16
    T = sum(lens)
    segs, o = [], 0
    for n in lens:
        segs.append((o, o + n))
        o += n
    q = (torch.nn.functional.normalize(torch.randn(T, H, dk), dim=-1) / dk ** 0.5).requires_grad_(True)
    k = torch.nn.functional.normalize(torch.randn(T, H, dk), dim=-1).requires_grad_(True)
    v = torch.randn(T, H, dv, requires_grad=True)
    g, beta = (-torch.rand(T, H)).requires_grad_(True), torch.rand(T, H, requires_grad=True)
    o1, S1 = gated_delta_chunked_varlen(q, k, v, g, beta, segs, chunk=C)
    ref = [gated_delta_chunked(q[a:b], k[a:b], v[a:b], g[a:b], beta[a:b], chunk=C) for a, b in segs]
    o2, S2 = torch.cat([r[0] for r in ref]), torch.stack([r[1] for r in ref])
    torch.testing.assert_close(o1, o2, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(S1, S2, atol=1e-5, rtol=1e-4)
    w = torch.randn_like(o1)
    g1 = torch.autograd.grad((o1 * w).sum() + S1.sum(), (q, k, v, g, beta))
    g2 = torch.autograd.grad((o2 * w).sum() + S2.sum(), (q, k, v, g, beta))
    for a, b in zip(g1, g2):
        torch.testing.assert_close(a, b, atol=1e-4, rtol=1e-4)


def test_packed_sequences_stay_independent():
    from axrl_b200.models.qwen3 import Qwen3Model
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    m = Qwen3Model(_cfg())
    m.init_weights(1)
    a, b = torch.randint(0, 1024, (37,)), torch.randint(0, 1024, (20,))
    both = m(torch.cat([a, b]), torch.cat([torch.arange(37), torch.arange(20)]).int(), causal_spec_from_cu_seqlens([0, 37, 57]))
    ha = m(a, torch.arange(37).int(), causal_spec_from_cu_seqlens([0, 37]))
    hb = m(b, torch.arange(20).int(), causal_spec_from_cu_seqlens([0, 20]))
    torch.testing.assert_close(both, torch.cat([ha, hb]), atol=1e-5, rtol=1e-4)


def test_hybrid_grpo_step_and_rollout_logprobs():
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine
    from axrl_b200.train.engine import TrainEngine
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer

    cfg = _cfg()
    wc = MegatronWorkerConfig(max_tokens_per_micro_batch=96, seed=3)
    wc.lr_scheduler.lr_warmup_steps = 0
    tr = TrainEngine(wc, cfg, "cpu")
    eng = RolloutEngine(tr.model, max_batch=4, kv_tokens=2048, max_context=256, use_cuda_graph=False, seed=1, burst=4)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(1, 1024, (n,), generator=g).tolist() for n in (9, 17, 9)]
    reqs = [GenRequest(rid=f"q{i}", prompt=p, max_new_tokens=12, temperature=1.0) for i, p in enumerate(prompts)]
    res = eng.generate(reqs)
    assert all(len(r.output_ids) == 12 for r in res)
    assert sorted(eng.gdn_free) == list(range(4))  # every state slot returned
    samples = [Sample.from_tokens(p, r.output_ids, rollout_logprobs=r.output_logprobs, advantage=float(i) - 1.0)
               for i, (p, r) in enumerate(zip(prompts, res))]
    batch = SampleBatch.from_samples(samples)
    lp = tr.compute_logprobs(batch)
    mask = batch["loss_mask"].bool()
    torch.testing.assert_close(lp[mask], batch["rollout_logprobs"][mask], atol=2e-4, rtol=1e-3)
    batch["old_logprobs"] = lp
    batch["ref_logprobs"] = lp
    before = {n: p.detach().clone() for n, p in tr.model.named_parameters() if "linear" not in n}
    m = tr.train_step(batch, GrpoTrainer(GrpoTrainerConfig(loss_type="grpo")))
    assert torch.isfinite(torch.tensor(m["grad_norm"])) and m["grad_norm"] > 0
    gdn = tr.model.layers[0].self_attn
    assert any(not torch.equal(p, before[n]) for n, p in tr.model.named_parameters() if n in before and ".self_attn.in_proj" in n)
    assert gdn.in_proj_qkv.shape[0] == gdn.conv_dim


def test_hybrid_checkpoint_and_hf_names_roundtrip():
    from axrl_b200.models.qwen3 import Qwen3Model, hf_state_dict, load_hf_state_dict
    from axrl_b200.sync.plan import qwen3_param_specs
    from axrl_b200.train.checkpoint import load_mcore_state_dict, mcore_state_dict

    cfg = _cfg()
    a, b = Qwen3Model(cfg), Qwen3Model(cfg)
    a.init_weights(4)
    b.init_weights(9)
    load_mcore_state_dict(b, mcore_state_dict(a))
    for (n, p), q in zip(a.named_parameters(), b.parameters()):
        torch.testing.assert_close(p, q, msg=n)
    c = Qwen3Model(cfg)
    c.init_weights(11)
    hf = {k: v.detach().clone() for k, v in hf_state_dict(a).items()}
    assert "model.layers.0.linear_attn.in_proj_qkv.weight" in hf and hf["model.layers.0.linear_attn.conv1d.weight"].dim() == 3
    load_hf_state_dict(c, hf)
    for (n, p), q in zip(a.named_parameters(), c.parameters()):
        torch.testing.assert_close(p, q, msg=n)
    names = {s.name for s in qwen3_param_specs(cfg)}
    assert names == {n for n, _ in a.named_parameters()}

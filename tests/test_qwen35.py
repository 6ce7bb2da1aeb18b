"""Qwen3.5-style hybrid MoE decoder (Gated DeltaNet + gated full attention with partial RoPE,
zero-centered RMSNorm, routed + shared experts) against the Hugging Face implementation.

The oracle is ``transformers``' ``Qwen3_5MoeForCausalLM`` in fp32 on the CPU (its PyTorch GDN
fallback); weights go through this package's HF loader, so names and layouts are checked too."""

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _hf_model(seed: int = 0):  # noqa: ANN202
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeForCausalLM

    cfg = Qwen3_5MoeTextConfig(vocab_size=512, hidden_size=128, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=32, linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16,
                               linear_value_head_dim=16, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                               shared_expert_intermediate_size=48)
    torch.manual_seed(seed)
    m = Qwen3_5MoeForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("A_log"):
                p.uniform_(-1.0, 1.0)
            elif p.dim() == 1:  # norm offsets, dt_bias
                p.normal_(0.0, 0.2)
            else:
                p.normal_(0.0, 0.08)
    return m, cfg


def _ours(hf, cfg):  # noqa: ANN001, ANN202
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model, load_hf_state_dict

    c = Qwen3Config.from_hf_dict(cfg.to_dict())
    assert c.attn_output_gate and c.zero_centered_norm and c.rotary_dim == 8 and c.is_hybrid and c.shared_expert_intermediate_size == 48
    m = Qwen3Model(c).float().eval()
    missing = load_hf_state_dict(m, {k: v.detach().clone() for k, v in hf.state_dict().items()})
    assert not missing
    return m


def test_logits_match_hf_packed_sequences():
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    hf, cfg = _hf_model()
    ours = _ours(hf, cfg)
    g = torch.Generator().manual_seed(1)
    lens = [37, 70]
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in lens]
    with torch.no_grad():
        ref = [hf(input_ids=s[None]).logits[0] for s in seqs]
        ids = torch.cat(seqs)
        pos = torch.cat([torch.arange(n) for n in lens])
        spec = causal_spec_from_cu_seqlens([0, lens[0], sum(lens)])
        got = ours.logits(ours(ids, pos, spec))
    want = torch.cat(ref)
    err = (got - want).abs().max().item()
    assert err < 2e-3 * max(1.0, want.abs().max().item()), err


def test_hf_and_megatron_round_trips():
    from axrl_b200.models.qwen3 import Qwen3Model, hf_state_dict, load_hf_state_dict
    from axrl_b200.train.checkpoint import load_mcore_state_dict, mcore_state_dict

    hf, cfg = _hf_model(seed=3)
    a = _ours(hf, cfg)
    # HF export: gated q_proj rows interleave [q_h; gate_h] per head; norms are offsets from 1
    ours_hf = hf_state_dict(a)
    ref = hf.state_dict()
    for k in ("model.layers.3.self_attn.q_proj.weight", "model.layers.3.self_attn.q_norm.weight", "model.norm.weight",
              "model.layers.0.input_layernorm.weight", "model.layers.1.mlp.shared_expert.down_proj.weight",
              "model.layers.2.mlp.shared_expert_gate.weight", "model.layers.0.linear_attn.conv1d.weight"):
        assert torch.allclose(ours_hf[k], ref[k], atol=1e-6, rtol=0), k  # norms: (w + 1) - 1
    F = cfg.moe_intermediate_size
    assert torch.equal(ours_hf["model.layers.1.mlp.experts.5.up_proj.weight"], ref["model.layers.1.mlp.experts.gate_up_proj"][5, F:])
    b = Qwen3Model(a.cfg).float()
    load_hf_state_dict(b, {k: v.detach().clone() for k, v in ours_hf.items()})
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.allclose(p, q, atol=1e-6, rtol=0), n
    # Megatron-Core layout round trip (zero-centered norms stored as offsets)
    sd = {k: v.clone() for k, v in mcore_state_dict(a).items()}
    assert torch.allclose(sd["decoder.final_layernorm.weight"], ref["model.norm.weight"], atol=1e-6)
    assert "decoder.layers.3.self_attention.linear_gate.weight" in sd and "decoder.layers.mlp.shared_experts.gate_weight" in sd
    c = Qwen3Model(a.cfg).float()
    load_mcore_state_dict(c, sd)
    for (n, p), (_, q) in zip(a.named_parameters(), c.named_parameters()):
        assert torch.allclose(p, q, atol=1e-6), n


def test_grpo_step_and_rollout_logprobs_on_cpu():
    """Rollout logprobs of the engine (gated attention, shared experts, GDN state slots) match the
    trainer's recomputation, and one GRPO step updates the new parameters."""
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine
    from axrl_b200.train.engine import TrainEngine
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer

    wc = MegatronWorkerConfig(max_tokens_per_micro_batch=96, seed=3)
    wc.lr_scheduler.lr_warmup_steps = 0
    tr = TrainEngine(wc, resolve_preset("tiny-qwen3.5"), "cpu")
    eng = RolloutEngine(tr.model, max_batch=4, kv_tokens=2048, max_context=256, use_cuda_graph=False, seed=1, burst=4)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(1, 1024, (n,), generator=g).tolist() for n in (9, 17)]
    res = eng.generate([GenRequest(rid=f"q{i}", prompt=p, max_new_tokens=10, temperature=1.0) for i, p in enumerate(prompts)])
    samples = [Sample.from_tokens(p, r.output_ids, rollout_logprobs=r.output_logprobs, advantage=float(i) - 0.5)
               for i, (p, r) in enumerate(zip(prompts, res))]
    batch = SampleBatch.from_samples(samples)
    lp = tr.compute_logprobs(batch)
    mask = batch["loss_mask"].bool()
    torch.testing.assert_close(lp[mask], batch["rollout_logprobs"][mask], atol=2e-4, rtol=1e-3)
    batch["old_logprobs"] = lp
    batch["ref_logprobs"] = lp
    names = ("layers.3.self_attn.attn_gate", "layers.0.mlp.shared_gate_up", "layers.1.mlp.shared_gate")
    before = {n: p.detach().clone() for n, p in tr.model.named_parameters() if n in names}
    m = tr.train_step(batch, GrpoTrainer(GrpoTrainerConfig(loss_type="grpo")))
    assert m["grad_norm"] > 0
    after = dict(tr.model.named_parameters())
    for n in names:
        assert not torch.equal(after[n], before[n]), n


def test_hf_checkpoint_directory_round_trip(tmp_path):
    """save_hf_checkpoint writes a Qwen3.5 text config and safetensors that load back unchanged."""
    import json

    from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
    from axrl_b200.train.checkpoint import hf_config, load_hf_checkpoint, save_hf_checkpoint

    a = Qwen3Model(resolve_preset("tiny-qwen3.5"))
    a.init_weights(7)
    save_hf_checkpoint(a, tmp_path, dtype=torch.float32)
    meta = json.loads((tmp_path / "config.json").read_text())
    assert meta["model_type"] == "qwen3_5_moe_text" and meta["rope_parameters"]["partial_rotary_factor"] == 0.25
    cfg = hf_config(tmp_path)
    assert cfg == a.cfg
    b = Qwen3Model(cfg)
    load_hf_checkpoint(b, tmp_path)
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.allclose(p, q, atol=1e-6, rtol=0), n

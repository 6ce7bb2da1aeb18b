"""Checkpoint formats: HF safetensors round trip, Megatron-style dist checkpoint round trip
(incl. optimizer state and the per-query-group QKV interleave), rotation and latest marker."""

import torch

from axrl_b200.configs import MegatronWorkerConfig
from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
from axrl_b200.train import checkpoint as ck
from axrl_b200.train.optimizer import FlatAdamW


def _model(seed):
    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16)
    m = Qwen3Model(cfg)
    m.init_weights(seed)
    return m


def test_hf_roundtrip(tmp_path):
    a, b = _model(1), _model(2)
    ck.save_hf_checkpoint(a, tmp_path, max_shard_bytes=50_000, dtype=torch.float32)
    assert (tmp_path / "model.safetensors.index.json").exists() and len(list(tmp_path.glob("*.safetensors"))) > 1
    ck.load_hf_checkpoint(b, tmp_path)
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.equal(p, q), n
    assert ck.hf_config(tmp_path).num_key_value_heads == 2


def test_qkv_interleave_inverse():
    w = torch.randn((8 + 2 * 4) * 16, 32)
    assert torch.equal(ck._qkv_from_mcore(ck._qkv_to_mcore(w, 8, 4, 16), 8, 4, 16), w)
    # group 0 of the Megatron layout = q heads 0..1, then k head 0, then v head 0
    m = ck._qkv_to_mcore(w, 8, 4, 16)
    assert torch.equal(m[:32], w[:32]) and torch.equal(m[32:48], w[128:144]) and torch.equal(m[48:64], w[192:208])


def test_dist_checkpoint_roundtrip_and_rotation(tmp_path):
    a, b = _model(1), _model(2)
    oa = FlatAdamW(a, MegatronWorkerConfig().optimizer, MegatronWorkerConfig().lr_scheduler)
    oa.exp_avg.normal_()
    oa.step_count = 7
    for step in (1, 2, 3):
        ck.save_dist_checkpoint(tmp_path, step, a, oa, extra={"dataset": {"x": step}}, most_recent_k=2)
    assert ck.latest_iteration(tmp_path) == 3
    assert sorted(p.name for p in tmp_path.glob("iter_*")) == ["iter_0000002", "iter_0000003"]
    assert (tmp_path / "iter_0000003" / ".metadata").exists()
    ob = FlatAdamW(b, MegatronWorkerConfig().optimizer, MegatronWorkerConfig().lr_scheduler)
    common = ck.load_dist_checkpoint(tmp_path, b, ob)
    assert common["extra"]["dataset"]["x"] == 3 and ob.step_count == 7
    assert torch.equal(ob.exp_avg, oa.exp_avg) and torch.equal(ob.master, oa.master)
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.equal(p, q), n
    keys = ck.mcore_state_dict(a)
    assert keys["decoder.layers.self_attention.linear_qkv.weight"].shape[0] == 2

"""Config tree: strict validation and YAML < CLI < env merge order."""

import pytest
import yaml

from axrl_b200.pipeline.config import PipelineExperimentConfig
from axrl_b200.utils.config_utils import config_to_args, load_and_validate_config, save_to_yaml


def test_defaults_and_paths():
    c = PipelineExperimentConfig()
    assert c.controller.run_mode == "online_rl_train"
    assert c.grpo.loss_type == "grpo2"
    assert c.megatron_worker.optimizer.lr == 1e-5
    assert c.megatron_worker.world_size() == 1


def test_merge_order(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text(yaml.safe_dump({"grpo": {"clip_ratio_high": 0.5, "loss_type": "tis"}, "megatron_worker": {"tp_size": 2}}))
    env = {"AXRL__megatron_worker__tp_size": "4", "AXRL__grpo__mismatch_token_clip_max": "2.0"}
    import os

    old = dict(os.environ)
    os.environ.update(env)
    try:
        c = load_and_validate_config(PipelineExperimentConfig, str(p), argv=["--grpo.clip_ratio_high=0.3", "--megatron_worker.tp_size=8",
                                                                            "--controller.colocated=false"])
    finally:
        os.environ.clear()
        os.environ.update(old)
    assert c.grpo.clip_ratio_high == 0.3  # CLI beats YAML
    assert c.grpo.loss_type == "tis"  # YAML kept
    assert c.megatron_worker.tp_size == 4  # env beats CLI
    assert c.grpo.mismatch_token_clip_max == 2.0
    assert c.controller.colocated is False


def test_strict_rejects_unknown(tmp_path):
    p = tmp_path / "bad.yaml"
    p.write_text(yaml.safe_dump({"grpo": {"no_such_field": 1}}))
    with pytest.raises(ValueError):
        load_and_validate_config(PipelineExperimentConfig, str(p), argv=[])


def test_roundtrip_yaml_and_args(tmp_path):
    c = PipelineExperimentConfig()
    p = tmp_path / "out.yaml"
    save_to_yaml(c, p)
    c2 = load_and_validate_config(PipelineExperimentConfig, str(p), argv=[], load_env_config=False)
    assert c2 == c
    args = config_to_args(c)
    assert args["--megatron_worker.optimizer.bf16"] == "true"
    assert args["--grpo.mismatch_token_clip_max"] == "null"


def test_opd_validation():
    from axrl_b200.configs import ModelConfig, OPDConfig

    with pytest.raises(ValueError):
        OPDConfig(enabled=True)
    OPDConfig(enabled=True, backend="megatron", teacher_model=ModelConfig(name="t"))

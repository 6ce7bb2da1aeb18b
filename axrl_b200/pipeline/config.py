"""Pipeline-level config: run modes and the experiment root.

Field paths match reference ``axrl/pipeline/config.py:19-82`` so that YAML and
``--controller.run_mode=...`` style overrides carry over unchanged.
"""

from __future__ import annotations

from typing import Literal

from axrl_b200.configs import (
    DatasetConfig,
    GrpoTrainerConfig,
    MegatronWorkerConfig,
    MetricLoggerConfig,
    MismatchTestConfig,
    ModelConfig,
    OnlineRLTrainConfig,
    RolloutWorkerConfig,
    SamplingConfig,
    SftTrainerConfig,
    StrictBaseModel,
)

PipelineRunMode = Literal["online_rl_train", "replay_rl_train", "eval_only", "sft_train", "mismatch_test"]


class ControllerConfig(StrictBaseModel):
    run_mode: PipelineRunMode = "online_rl_train"
    output_dir_name: str = "grpo"
    colocated: bool = True
    num_rollout_actors: int = 16
    num_cpus_per_actor: int = 4
    max_running_requests: int = 256
    smoke_eval_rollouts: int | None = None
    save_eval_rollouts: bool = True
    allow_prefix_merging: bool = True


class EvalOnlyConfig(StrictBaseModel):
    model: ModelConfig | None = None


class ReplayRLTrainConfig(StrictBaseModel):
    sample_dict_path: str | None = None
    rollout_groups_path: str | None = None


class PipelineExperimentConfig(StrictBaseModel):
    controller: ControllerConfig = ControllerConfig()
    eval_only: EvalOnlyConfig = EvalOnlyConfig()
    megatron_worker: MegatronWorkerConfig = MegatronWorkerConfig()
    value_worker: MegatronWorkerConfig | None = None
    rollout_worker: RolloutWorkerConfig = RolloutWorkerConfig()
    train_datasets: list[DatasetConfig] | None = None
    test_datasets: list[DatasetConfig] | None = None
    eval_sampling_config: SamplingConfig = SamplingConfig()
    train_sampling_config: SamplingConfig = SamplingConfig()
    grpo: GrpoTrainerConfig = GrpoTrainerConfig()
    sft: SftTrainerConfig = SftTrainerConfig()
    online_rl_train: OnlineRLTrainConfig = OnlineRLTrainConfig()
    replay_rl_train: ReplayRLTrainConfig = ReplayRLTrainConfig()
    mismatch_test: MismatchTestConfig = MismatchTestConfig()
    logger: MetricLoggerConfig = MetricLoggerConfig()

"""Strict, typed configuration tree.

Class names and field paths intentionally match the reference's public config
surface (``axrl/configs.py:62-658``) so existing YAML files and
``--path.to.field=value`` overrides keep working.  Megatron-specific knobs are
interpreted by this framework's own trainer (``axrl_b200.train``) instead of
Megatron-Core.

Directory defaults come from ``AXRL_*`` environment variables (reference
``axrl/configs.py:20-44``); nothing here touches the filesystem at import time.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path
from typing import Literal

from pydantic import BaseModel, ConfigDict, field_validator


@dataclass
class DirInfo:
    data: Path
    model: Path
    output: Path
    log: Path


def _dirs_from_env() -> DirInfo:
    root = Path.home() / "axrl-data"
    out = Path(os.environ.get("AXRL_OUTPUT_DIR", str(root / "outputs" / os.environ.get("AXRL_OUTPUT_DIR_NAME", "default"))))
    return DirInfo(
        data=Path(os.environ.get("AXRL_DATA_DIR", str(root / "datasets"))),
        model=Path(os.environ.get("AXRL_MODEL_DIR", str(root / "models"))),
        output=out,
        log=Path(os.environ.get("AXRL_LOG_DIR", str(out / "logs"))),
    )


AXRL_DIR = _dirs_from_env()
STABLE_MODEL_DIR = Path(os.environ.get("AXRL_STABLE_MODEL_DIR", str(AXRL_DIR.model)))
SHARED_MODEL_DIR = Path(os.environ.get("AXRL_SHARED_MODEL_DIR", str(AXRL_DIR.model / "shared_models")))
RAY_TASK_QUEUE_MAX_CONCURRENCY = 8192
IGNORE_INDEX: int = -100


def resolve_model_name(model_name: str) -> str:
    """Absolute names pass through; otherwise prefer the stable dir, then the shared dir."""
    p = Path(model_name)
    if p.is_absolute() or (STABLE_MODEL_DIR / p).exists():
        return model_name
    shared = SHARED_MODEL_DIR / p
    return str(shared.absolute()) if shared.exists() else model_name


class StrictBaseModel(BaseModel):
    """Pydantic base that rejects unknown fields (typos in YAML fail loudly)."""

    model_config = ConfigDict(extra="forbid")


LogLevel = Literal["debug", "info", "warning", "error", "critical"]
ValueAggType = Literal[
    "token-mean", "seq-mean-token-mean", "seq-mean-token-std", "token-max", "token-min", "token-std", "token-p05", "token-p95"
]
SampleType = Literal["uniform", "uniform-no-easy", "low-success-rate", "intermediate-success-rate"]
Role = Literal["user", "assistant", "system", "tool"]
PlacementGroupStrategy = Literal["PACK", "SPREAD", "STRICT_PACK", "STRICT_SPREAD"]
MetricLoggerType = Literal["tensorboard", "wandb", "console"]


class RolloutSamplerConfig(StrictBaseModel):
    sample_type: SampleType = "uniform"
    epsilon: float = 0.05


class LoggerConfig(StrictBaseModel):
    name: str = "axrl"
    level: LogLevel = "info"


class MetricLoggerConfig(StrictBaseModel):
    logger_type: MetricLoggerType = "console"
    name: str = "main-process"
    group_name: str = "default_group"
    project_name: str = "axrl"
    run_id: str | None = None

    def get_log_dir(self) -> Path:
        return AXRL_DIR.log.absolute()


class DatasetConfig(StrictBaseModel):
    name: str
    data_path: str | None = None
    eval_num_rollouts_per_prompt: int | None = None
    subset_key: str | None = None


class HfDataConfig(StrictBaseModel):
    repo_id: str = "open-r1/DAPO-Math-17k-Processed"
    filename: str = "all/train-00000-of-00001.parquet"

    def get_full_path(self) -> Path:
        return (AXRL_DIR.data / self.repo_id / self.filename).absolute()


class ModelConfig(StrictBaseModel):
    """Model identity.  ``name`` is an HF repo id / local dir, or a built-in
    architecture preset such as ``"synthetic:qwen3-8b"`` (random init)."""

    name: str = "Qwen/Qwen3-0.6B-Base"
    trust_remote_code: bool = True
    seq_length: int = 2048

    def get_full_path(self) -> Path:
        resolved = Path(resolve_model_name(self.name))
        return resolved if resolved.is_absolute() else (AXRL_DIR.model / self.name).absolute()


class WorkerConfig(StrictBaseModel):
    name: str = "default-worker"


class InferWorkerConfig(WorkerConfig):
    pass


class SamplingConfig(StrictBaseModel):
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    repetition_penalty: float = 1.0
    max_total_tokens: int = 4096
    max_new_tokens: int | None = None
    stop: list[str] | str | None = None


class OAIClientConfig(InferWorkerConfig):
    """HTTP generation client (token ids in, token-aligned logprobs out)."""

    base_url: str
    sampling_config: SamplingConfig = SamplingConfig()
    request_timeout_seconds: float | None = None
    max_connections: int | None = 512
    max_keepalive_connections: int | None = 128
    retry_initial_sleep_seconds: float = 1.0
    retry_max_sleep_seconds: float = 30.0


# The reference only knows "sglang"; here the rollout engine is this package's
# own paged-KV engine.  "sglang" is accepted as an alias so old YAML validates.
EngineType = Literal["axrl", "sglang"]


class RolloutWorkerConfig(InferWorkerConfig):
    engine_type: EngineType = "axrl"
    model: ModelConfig = ModelConfig()
    sampling_config: SamplingConfig = SamplingConfig()
    gpu_memory_utilization: float = 0.6
    dp_size: int = 1
    tp_size: int = 2
    pp_size: int = 1
    ep_size: int = 1
    moe_a2a_backend: Literal["none", "deepep", "mooncake", "mori", "ascend_fuseep", "flashinfer"] = "none"
    moe_runner_backend: str | None = None
    enable_routing_replay: bool = False
    num_workers: int = 1
    clear_partial_outputs_after_abort: bool = False
    continue_generation_after_abort: bool = True
    log_level: LogLevel = "info"
    max_running_requests: int = 128
    max_running_requests_eval: int | None = None
    max_num_batched_tokens: int | None = None
    load_dummy_weights: bool = False
    attention_backend: str | None = None
    kv_cache_dtype: Literal["auto", "fp8_e4m3", "fp8_e5m2"] = "auto"
    prefill_max_requests: int | None = None
    enable_fp32_lm_head: bool = True
    enable_metrics: bool = True
    dtype: Literal["auto", "float16", "bfloat16"] = "bfloat16"
    master_addr: str = "127.0.0.1"
    master_port: int = 20250
    nnodes: int = 1
    node_rank: int = 0
    max_imbalance: int = 16
    # B200 engine knobs (no reference counterpart): paged-KV page size and
    # whether the decode step is captured in a CUDA graph.
    kv_page_size: int = 64
    use_cuda_graph: bool = True
    weight_dtype: Literal["bf16", "fp8_block"] = "bf16"

    @field_validator("kv_cache_dtype")
    @classmethod
    def _kv_dtype_supported(cls, v: str) -> str:
        # The paged KV cache and its decode kernel are bf16; an fp8 cache would be accepted and
        # silently stored in bf16, so it is rejected instead.
        if v != "auto":
            raise ValueError(f"kv_cache_dtype={v!r} is not supported by the rollout engine (bf16 KV cache only); use 'auto'")
        return v

    def gpus_per_worker(self) -> int:
        return self.tp_size * self.pp_size


TeacherBackend = Literal["sglang", "megatron"]
OPDStudentLogprobSource = Literal["rollout_logprobs", "old_logprobs", "cur_logprobs"]


class OPDConfig(StrictBaseModel):
    """On-policy distillation (reference ``axrl/configs.py:246-277``)."""

    enabled: bool = False
    backend: TeacherBackend = "sglang"
    teacher_model: ModelConfig | None = None
    sglang_worker: RolloutWorkerConfig = RolloutWorkerConfig()
    sglang_host: str | None = None
    sglang_port: int | None = None
    opd_alpha: float = 0.1
    reverse_kl_clip: float | None = 10.0
    student_logprob_source: OPDStudentLogprobSource = "cur_logprobs"
    normalize_student_logprob_scale: bool = False
    teacher_weight_name: str = "opd_teacher_weights"

    def model_post_init(self, __context: object, /) -> None:
        if not self.enabled:
            return
        if not 0.0 <= self.opd_alpha <= 1.0:
            raise ValueError("OPD opd_alpha must lie in [0, 1].")
        if self.teacher_model is None:
            raise ValueError("OPD requires teacher_model when enabled.")
        if self.backend == "sglang":
            if self.sglang_worker.model != self.teacher_model:
                raise ValueError("OPD engine teacher model must equal sglang_worker.model.")
            if self.sglang_port is None:
                raise ValueError("OPD engine backend requires sglang_port.")
        elif not self.teacher_weight_name:
            raise ValueError("OPD trainer backend requires a teacher_weight_name.")


class DataloaderConfig(StrictBaseModel):
    num_workers: int = 4


class GradSpikeDebugConfig(StrictBaseModel):
    """Grad-norm spike snapshotting: a spike is ``norm > spike_ratio * median(last history_window)``."""

    enabled: bool = False
    warmup_steps: int = 10
    spike_ratio: float = 2.0
    history_window: int = 100
    max_snapshots: int = 3
    save_per_param_grads: bool = True


class MCoreOptimizerConfig(StrictBaseModel):
    optimizer: str = "adam"
    lr: float | None = None
    min_lr: float | None = None
    weight_decay: float = 0.01
    use_distributed_optimizer: bool = True
    clip_grad: float = 1.0
    fp16: bool = False
    bf16: bool = False
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    optimizer_cpu_offload: bool = False
    optimizer_offload_fraction: float = 0.0
    use_stateless_adam: bool = False
    adam_eps: float = 1e-8


class MCoreLrSchedulerConfig(StrictBaseModel):
    init_lr: float = 1e-5
    max_lr: float = 1e-5
    min_lr: float = 1e-6
    lr_warmup_steps: int = 100
    lr_decay_steps: int = 1000000
    lr_decay_style: Literal["constant", "cosine", "linear"] = "constant"
    start_wd: float = 0.01
    end_wd: float = 0.01
    wd_incr_steps: int = 1000000
    wd_incr_style: Literal["constant", "cosine", "linear"] = "constant"
    use_checkpoint_opt_param_scheduler: bool | None = True
    override_opt_param_scheduler: bool | None = False
    wsd_decay_steps: int | None = None
    lr_wsd_decay_style: str | None = None


TrainerType = Literal["sft"]
MegatronModelRole = Literal["actor", "value"]


class SftTrainerConfig(StrictBaseModel):
    compute_accuracy: bool = False
    compute_entropy: bool = False


SFTConfig = SftTrainerConfig


class MegatronWorkerConfig(StrictBaseModel):
    """Trainer worker config.  The name is kept for YAML compatibility; the
    engine behind it is ``axrl_b200.train`` (TP/PP/CP/EP/DP on B200)."""

    model: ModelConfig = ModelConfig()
    model_role: MegatronModelRole = "actor"
    seed: int = 42
    tp_size: int = 1
    pp_size: int = 1
    vpp_size: int | None = None
    dp_size: int = 1
    cp_size: int = 1
    ep_size: int = 1
    etp_size: int | None = 1
    distributed_timeout_seconds: int = 1800
    enable_routing_replay: bool = False
    replay_routing_for_loss_tokens_only: bool = False
    fp8: Literal["e4m3", "hybrid"] | None = None
    fp8_recipe: Literal["tensorwise", "delayed", "mxfp8", "blockwise", "custom"] = "blockwise"
    data_loader: DataloaderConfig = DataloaderConfig()
    padding_sample_length: int = 4
    train_micro_batch_size: int = 4
    eval_micro_batch_size: int = 8
    global_batch_size: int = 32
    use_dynamic_batch_size: bool = True
    num_epochs: int = 100
    moe_aux_loss_coeff: float = 0
    moe_router_load_balancing_type: Literal["none", "aux_loss", "seq_aux_loss", "global_aux_loss", "sinkhorn"] = "none"
    recompute_granularity: Literal["full", "selective"] | None = None
    recompute_method: Literal["uniform", "block"] | None = None
    recompute_num_layers: int | None = None
    recompute_modules: list[str] | None = None
    cpu_offloading: bool = False
    cpu_offloading_num_layers: int = 0
    cpu_offloading_double_buffering: bool = False
    log_every_k_steps: int = 10
    checkpoint_dir: str = "checkpoints/megatron"
    checkpoint_step: int | None = None
    most_recent_checkpoint_k: int = 2
    save_hf_checkpoint: bool = False
    reset_init_weights_every_k_steps: int | None = None
    log_microbatches: bool = False
    log_gpu_usaegs: bool = False
    metric_logger_config: MetricLoggerConfig = MetricLoggerConfig()
    log_level: LogLevel = "info"
    fp16: bool = False
    bf16: bool = True
    use_gloo_process_groups: bool = True
    apply_rope_fusion: bool | None = None
    attention_backend: str | None = "flash"
    deterministic_mode: bool = True
    batch_invariant_mode: bool = False
    use_language_model_only: bool = False
    spike_debug: GradSpikeDebugConfig = GradSpikeDebugConfig()
    optimizer: MCoreOptimizerConfig = MCoreOptimizerConfig(lr=1e-5, min_lr=1e-6, bf16=True, use_distributed_optimizer=True)
    lr_scheduler: MCoreLrSchedulerConfig = MCoreLrSchedulerConfig()
    num_dataloader_workers: int = 0
    inference_only: bool = False
    shuffle_train_data: bool = False
    enable_fp32_lm_head: bool = False
    use_magi_merged_forward: bool = False
    use_magi_flat_forward: bool = False
    # Max tokens per packed micro-batch when use_dynamic_batch_size is on.
    max_tokens_per_micro_batch: int = 16384

    @field_validator("fp8")
    @classmethod
    def _fp8_training_supported(cls, v: str | None) -> str | None:
        # fp8 serves the rollout (RolloutWorkerConfig.weight_dtype="fp8_block"); the trainer's GEMMs
        # are bf16, so an fp8 training recipe is rejected rather than ignored.
        if v is not None:
            raise ValueError(f"fp8={v!r} training is not supported (bf16 training; fp8 is available for rollout weights)")
        return v

    def world_size(self) -> int:
        return self.dp_size * self.tp_size * self.pp_size * self.cp_size

    def expert_tensor_parallel_size(self) -> int:
        return self.tp_size if self.etp_size is None else self.etp_size

    def expert_parallel_group_size(self) -> int:
        return self.expert_tensor_parallel_size() * self.ep_size * self.pp_size

    def get_checkpoint_dir(self) -> Path:
        return (AXRL_DIR.output / self.checkpoint_dir).absolute()


class EntropyControlConfig(StrictBaseModel):
    target_entropy: float = 0.1
    alpha: float = 0.0
    compute_entropy: bool = False
    top_k: int = -1
    top_quantile: float = 1.0
    easy_score_cutoff: float = 0.4
    epsilon: float = 1e-6


RewardMeanType = Literal["group"]
RewardStdType = Literal["group"]
LossType = Literal["grpo", "ppo", "tis", "gspo", "grpo2", "topr", "kimi2_5"]
IsBaseLogprobsType = Literal["old_logprobs", "rollout_logprobs"]
KlBaseLogprobsType = Literal["old_logprobs", "ref_logprobs"]
MicroBatchDenominatorType = Literal["token", "sequence", "seq_turn"]


class PPOValueConfig(StrictBaseModel):
    gamma: float = 1.0
    gae_lambda: float = 1.0
    value_clip: float | None = 0.2
    value_loss_coef: float = 1.0
    num_value_only_updates: int = 0
    use_stateless_value_model: bool = False


class GrpoTrainerConfig(StrictBaseModel):
    loss_type: LossType = "grpo2"
    clip_ratio_high: float = 0.28
    clip_ratio_low: float = 0.2
    dual_clip_neg_adv_factor: float | None = 3.0
    dual_soft_clip: float | None = 3
    log_sample: bool = True
    normalize_advantage_by_batch_std: bool = False
    loss_agg_type: ValueAggType = "token-mean"
    micro_batch_denominator_type: MicroBatchDenominatorType = "token"
    entropy_control: EntropyControlConfig = EntropyControlConfig()
    kl_control_alpha: float = 0.0
    is_base_logprobs: IsBaseLogprobsType = "old_logprobs"
    kl_base_logprobs: KlBaseLogprobsType = "old_logprobs"
    mismatch_token_clip_max: float | None = None
    mismatch_seq_masking_low: float | None = None
    mismatch_seq_masking_high: float | None = None
    mismatch_token_veto_threshold: float | None = None
    icepop_masking_low: float | None = None
    icepop_masking_high: float | None = None
    turn_reward_alpha: float = 0.0
    seq_turn_alpha: float | None = None
    opd: OPDConfig = OPDConfig()
    normalize_advantages_over_valid_tokens_in_batch: bool = False
    ppo_value: PPOValueConfig | None = None


class OnlineRLTrainConfig(StrictBaseModel):
    eval_on_start: bool = True
    num_rollouts_per_conversation: int = 8
    model_sync_every_n_global_updates: int = 4
    checkpoint_every_n_global_updates: int | None = 1024
    eval_every_n_global_updates: int = 16
    batch_rollout_for_n_global_updates: int = 4
    max_global_updates: int = 4000
    strict_on_policy: bool = False
    reward_mean_type: RewardMeanType = "group"
    reward_std_type: RewardStdType = "group"
    reward_history_size: int = 64
    sample_type: SampleType = "uniform"
    filter_zero_std: bool = False
    max_prompt_length: int | None = None
    sort_sampled_prompts_by_response_length: bool = True
    rollout_save_filename: str = "valid_rollouts"
    rollout_save_every_n_global_updates: int | None = None
    save_all_rollouts: bool = False


class GrpoConfig(GrpoTrainerConfig):
    """Combined GRPO + loop config used by the legacy controller."""

    eval_on_start: bool = True
    num_rollouts_per_conversation: int = 16
    model_sync_every_n_global_updates: int = 4
    checkpoint_every_n_global_updates: int = 1024
    eval_every_n_global_updates: int = 64
    batch_rollout_for_n_global_updates: int = 8
    max_global_updates: int = 2000
    strict_on_policy: bool = False
    reward_mean_type: RewardMeanType = "group"
    reward_std_type: RewardStdType = "group"
    reward_history_size: int = 64
    sample_type: SampleType = "uniform"
    filter_zero_std: bool = False
    max_prompt_length: int | None = None
    sort_sampled_prompts_by_response_length: bool = True
    rollout_save_filename: str = "valid_rollouts"
    rollout_save_every_n_global_updates: int | None = None
    save_all_rollouts: bool = False


class MismatchTestConfig(StrictBaseModel):
    enabled: bool = False
    name: str = "cur-exp"
    output_dir: str = "tmp/mismatch-test"
    override_rollouts_if_exists: bool = False
    baseline_samples_path: str | None = None
    baseline_name: str | None = None

    @staticmethod
    def _sanitize_name(name: str) -> str:
        return name.replace("/", "_")

    def get_output_dir(self) -> Path:
        return Path(self.output_dir)

    def get_result_dir(self) -> Path:
        return self.get_output_dir() / "results"

    def get_data_root(self) -> Path:
        return self.get_result_dir() / "data"

    def get_log_dir(self) -> Path:
        return self.get_result_dir() / "log"

    def get_fig_dir(self) -> Path:
        return self.get_result_dir() / "figs"

    def get_exp_data_dir(self, name: str) -> Path:
        return self.get_data_root() / self._sanitize_name(name)

    def get_valid_rollouts_path(self, name: str) -> Path:
        return self.get_exp_data_dir(name) / f"valid_rollouts-{self._sanitize_name(name)}.zst"

    def get_training_samples_path(self, name: str) -> Path:
        return self.get_exp_data_dir(name) / f"training_samples-{self._sanitize_name(name)}.zst"

    def get_result_path(self, name: str) -> Path:
        return self.get_log_dir() / f"{self._sanitize_name(name)}.zst"

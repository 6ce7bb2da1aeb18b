"""Spike detection/snapshot/replay on CPU (tiny model) and trainer-side OPD teacher annotation."""

import torch

from axrl_b200.configs import GradSpikeDebugConfig, GrpoTrainerConfig, MegatronWorkerConfig
from axrl_b200.data.sample import Sample, SampleBatch
from axrl_b200.models.qwen3 import resolve_preset
from axrl_b200.train.engine import TrainEngine
from axrl_b200.train.spike_debug import SpikeDetector, replay_snapshot, save_spike_snapshot
from axrl_b200.trainer.grpo_trainer import GrpoTrainer


def test_detector():
    d = SpikeDetector(GradSpikeDebugConfig(enabled=True, warmup_steps=3, spike_ratio=2.0, history_window=10))
    flags = [d.observe(x) for x in [1, 1, 1, 1, 1.1, 5.0, 1.0]]
    assert flags == [False, False, False, False, False, True, False]


def _batch():
    torch.manual_seed(0)
    ss = [Sample.from_tokens(list(range(1, 9)), [5, 6, 7, 8], advantage=a, rollout_logprobs=[-1.0] * 4) for a in (1.0, -1.0)]
    b = SampleBatch.from_samples(ss)
    b["old_logprobs"] = b["rollout_logprobs"].clone()
    b["ref_logprobs"] = b["rollout_logprobs"].clone()
    return b


def test_snapshot_replay(tmp_path):
    eng = TrainEngine(MegatronWorkerConfig(), resolve_preset("tiny"), "cpu")
    tr = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo"))
    b = _batch()
    m = eng.train_step(b, tr)
    d = save_spike_snapshot(tmp_path, 5, m["grad_norm"], eng, b, GradSpikeDebugConfig(enabled=True))
    before = eng.optim.master.clone()
    r = replay_snapshot(d, eng, tr)
    assert torch.equal(eng.optim.master, before)
    assert abs(r["replayed_grad_norm"] - r["recorded_grad_norm"]) / r["recorded_grad_norm"] < 0.5


def test_engine_teacher_annotation():
    from axrl_b200.opd.teacher_logprobs import annotate_engine_teacher_logprobs

    eng = TrainEngine(MegatronWorkerConfig(inference_only=True), resolve_preset("tiny"), "cpu")
    b = _batch()
    teacher = eng.snapshot_weights() * 1.5
    student_before = eng.snapshot_weights()
    annotate_engine_teacher_logprobs(b, eng, teacher)
    assert "teacher_logprobs" in b and torch.equal(eng.snapshot_weights(), student_before)
    own = eng.compute_logprobs(b)
    assert not torch.allclose(own, b["teacher_logprobs"])

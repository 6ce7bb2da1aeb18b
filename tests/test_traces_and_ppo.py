"""Multi-turn traces (turn samples, packing, compaction, R3 rows), PPO GAE / value loss, SFT loss,
and the trajectory-grouped global batch iterator."""

import numpy as np
import pytest
import torch

from axrl_b200.data.global_batch_iterator import build_global_batches_for_dp_rank
from axrl_b200.data.rollout_trace import RolloutTrace, pack_rollout_traces_for_train_batches
from axrl_b200.data.sample import SampleBatch
from axrl_b200.trainer.ppo_utils import build_terminal_token_rewards, clipped_value_loss_per_token, compute_gae


def _trace(turns=3, boundary=None):
    t = RolloutTrace(assistant_boundary_token_id=boundary)
    t.initialize([1, 2, 3, 4])
    for k in range(turns):
        t.append_assistant([10 + k, 20 + k, 30 + k], [-0.1, -0.2, -0.3])
        if k < turns - 1:
            t.append_user_or_tool_message([100 + k, 101 + k])
    return t


def test_turn_samples_and_labels():
    t = _trace()
    assert len(t.turn_samples) == 3
    s = t.turn_samples[1]
    n = len(s.input_ids)
    assert s.loss_mask.sum() == 3 and s.labels[n - 2] == 31 and s.labels[n - 1] == -100
    assert np.allclose(s.rollout_logprobs[s.loss_mask], [-0.1, -0.2, -0.3])
    assert t.token_trace.num_assistant_turns == 3


def test_packed_samples_cover_all_trainable_tokens():
    t = _trace(4)
    for s in t.turn_samples:
        s.advantage = np.where(s.loss_mask, 1.0, 0.0).astype(np.float32)
    big = t.to_packed_samples(10_000)
    assert len(big) == 1 and big[0].loss_mask.sum() == 12
    exact = t.to_packed_samples(22)  # the longest turn sample is 22 tokens: the linear chain fits exactly
    assert len(exact) == 1 and int(exact[0].loss_mask.sum()) == 12
    with pytest.raises(ValueError):
        t.to_packed_samples(21)
    flat = t.to_packed_samples(10_000, allow_prefix_sharing=False)
    assert len(flat) == 1 and flat[0].merge_info is None and flat[0].loss_mask.sum() == 12


def test_boundary_token_and_routing_rows():
    t = RolloutTrace(assistant_boundary_token_id=99)
    t.initialize([1, 2, 3])
    t.append_assistant([5, 6], [0, 0], routing_handle="h0")
    assert t.token_trace.routing_row_count_per_handle == [4]  # 5 tokens -> 4 rows
    t.append_user_or_tool_message([7])
    t.append_assistant([8, 99], [0, 0], routing_handle="h1")
    assert t.token_ids.tolist() == [1, 2, 3, 5, 6, 99, 7, 8, 99]
    assert t.token_trace.captured_routing_rows == 8


def test_compaction_drops_stale_handles():
    t = RolloutTrace()
    t.initialize([1, 2])
    t.append_assistant([3], [0], routing_handle="a")
    t.append_user_or_tool_message([50, 51, 52])
    t.append_assistant([4], [0], routing_handle="b")
    t.append_user_or_tool_message([60, 61])
    t.append_assistant([5], [0], routing_handle="c")
    t.compact(max_recent_tool_results=1, placeholder_ids=[0])
    assert t.routing_handles == ["a"]
    assert t.token_ids.tolist() == [1, 2, 3, 0, 4, 60, 61, 5]


def test_pack_traces_keeps_trajectory_ids():
    traces = [_trace(2), _trace(3)]
    out = pack_rollout_traces_for_train_batches(traces, 10_000)
    assert sorted({s.trajectory_id for s in out}) == [0, 1]


def test_gae_and_value_loss():
    rewards = build_terminal_token_rewards(torch.tensor([1.0, 2.0]), torch.tensor([[0, 1, 1, 0], [1, 1, 1, 1]]).bool())
    assert rewards.tolist() == [[0, 0, 1, 0], [0, 0, 0, 2]]
    values = torch.tensor([[0.0, 0.5, 0.5, 0.0], [0.1, 0.2, 0.3, 0.4]])
    mask = torch.tensor([[0, 1, 1, 0], [1, 1, 1, 1]]).bool()
    adv, ret = compute_gae(rewards, values, mask, gamma=1.0, gae_lambda=1.0)
    assert adv[0].tolist() == pytest.approx([0, 0.5, 0.5, 0])
    assert ret[1].tolist() == pytest.approx([2, 2, 2, 2])
    loss, cf = clipped_value_loss_per_token(torch.tensor([[1.5]]), torch.tensor([[1.0]]), torch.tensor([[2.0]]), value_clip=0.2)
    assert loss.item() == pytest.approx(0.64) and cf.item() == 1.0


def test_sft_loss():
    from axrl_b200.configs import SftTrainerConfig
    from axrl_b200.trainer.sft_trainer import SftTrainer

    lp = torch.tensor([[-1.0, -3.0, 0.0]])
    loss, denom, m = SftTrainer(SftTrainerConfig()).loss_func({"log_prob": lp}, {"loss_mask": torch.tensor([[True, True, False]]), "labels": lp})
    assert loss.item() == pytest.approx(2.0) and int(denom) == 2


def test_global_batches_dp_slices():
    from axrl_b200.data.sample import Sample

    samples = [Sample.from_tokens([1, 2, 3], [4, 5], trajectory_id=i // 2) for i in range(10)]  # 5 trajectories
    batch = SampleBatch.from_samples(samples)
    slices = [build_global_batches_for_dp_rank(batch, global_batch_size=5, dp_size=4, dp_rank=r) for r in range(4)]
    rows = sum(len(s[0]) for s in slices)
    assert rows == 12  # 10 rows padded to a multiple of 4
    assert sum(int((s[0]["index"] == -1).sum()) for s in slices) == 2

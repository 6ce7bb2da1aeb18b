"""Trajectory-grouped global batches with DP padding and round-robin DP slicing.

Reference: ``axrl/data/global_batch_iterator.py:42-173``.  All packed samples of one
trajectory land in the same global batch (so gradient magnitude does not depend on how
a long trajectory was split), the batch is padded with zero-loss rows to a multiple of
the DP size, optionally shuffled with a per-batch seed, and dealt round-robin to ranks.
"""

from __future__ import annotations

import torch

from axrl_b200.data.sample import SampleBatch, make_padding_samples, tensorize_samples


def assert_trajectory_count_divisible(samples: SampleBatch, global_batch_size: int) -> int:
    tid = samples["trajectory_id"]
    assert int(tid.min()) >= 0, "training samples need non-negative trajectory_id"
    n = int(tid.max()) + 1
    assert n % global_batch_size == 0, f"num_trajectories ({n}) must be divisible by global_batch_size ({global_batch_size})"
    return n


def group_rows_by_global_batch(trajectory_ids: list[int], global_batch_size: int) -> list[list[int]]:
    assert global_batch_size > 0
    if not trajectory_ids:
        return []
    n = max(trajectory_ids) + 1
    assert min(trajectory_ids) >= 0 and set(trajectory_ids) == set(range(n)), "trajectory ids must be contiguous from 0"
    out: list[list[int]] = [[] for _ in range(-(-n // global_batch_size))]
    for row, t in enumerate(trajectory_ids):
        out[t // global_batch_size].append(row)
    return out


def pad_to_dp_multiple(batch: SampleBatch, dp_size: int, padding_sample_length: int) -> SampleBatch:
    rem = len(batch) % dp_size
    if rem == 0:
        return batch
    pad = tensorize_samples(make_padding_samples(dp_size - rem, padding_sample_length))
    pad.tensors["index"].fill_(-1)
    for k in list(pad.tensors):
        if k not in batch.tensors:
            del pad.tensors[k]
    for k in batch.tensors:
        if k not in pad.tensors:
            pad.tensors[k] = torch.zeros((len(pad), *batch.tensors[k].shape[1:]), dtype=batch.tensors[k].dtype)
    pad.objects = {k: [None] * len(pad) for k in batch.objects}
    return SampleBatch.concat([batch, pad])


def build_global_batches_for_dp_rank(samples: SampleBatch, *, global_batch_size: int, dp_size: int, dp_rank: int,
                                     padding_sample_length: int = 4, shuffle: bool = False, shuffle_seed: int = 0) -> list[SampleBatch]:
    assert 0 <= dp_rank < dp_size
    tids = samples["trajectory_id"].tolist()
    if all(t == -1 for t in tids):
        tids = list(range(len(tids)))
    out = []
    for gb, rows in enumerate(group_rows_by_global_batch(tids, global_batch_size)):
        assert rows, f"global batch {gb} is empty"
        b = pad_to_dp_multiple(samples.select_rows(rows), dp_size, padding_sample_length)
        perm = torch.randperm(len(b), generator=torch.Generator().manual_seed(shuffle_seed + gb)).tolist() if shuffle else list(range(len(b)))
        out.append(b.select_rows(perm[dp_rank::dp_size]))
    return out

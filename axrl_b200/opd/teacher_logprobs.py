"""On-policy distillation: teacher log-probs for training samples.

Reference: ``annotate_sglang_teacher_logprobs`` (HTTP teacher, ``axrl/opd/teacher_logprobs.py:80-117``)
and the trainer-side path that swaps a CPU weight snapshot of the teacher into the model
(``axrl/worker/megatron_worker.py:1372-1385``).  The resulting ``teacher_logprobs`` feed
``GrpoTrainer.apply_opd_to_advantages``.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from axrl_b200.data.sample import Sample, SampleBatch


def annotate_engine_teacher_logprobs(batch: SampleBatch, train_engine: Any, teacher_weights: torch.Tensor, temperature: float = 1.0) -> None:
    """Swap the teacher's flat weights in, compute per-token log-probs, swap the student back."""
    cur = train_engine.snapshot_weights()
    try:
        train_engine.load_weights(teacher_weights)
        batch["teacher_logprobs"] = train_engine.compute_logprobs(batch, temperature)
    finally:
        train_engine.load_weights(cur)


async def annotate_http_teacher_logprobs(samples: list[Sample], client: Any) -> None:
    """Score each sample's trainable tokens with a served teacher (``GenerationClient.score``)."""
    for s in samples:
        n = int(s.attention_mask.sum())
        idx = np.flatnonzero(s.loss_mask)
        if idx.size == 0:
            s.teacher_logprobs = np.zeros(len(s.input_ids), np.float32)
            continue
        start = int(idx[0])
        lps = await client.score(s.input_ids[:n].tolist(), start)
        out = np.zeros(len(s.input_ids), np.float32)
        out[start:start + len(lps)] = lps[: n - 1 - start]
        s.teacher_logprobs = out

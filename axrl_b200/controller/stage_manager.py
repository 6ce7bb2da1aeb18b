"""Placement stage machines for colocated and disaggregated deployments.

Reference: ``ColocatedStageManager`` / ``DisaggregatedStageManager``
(``axrl/controller/stage_manager.py:27-110``).  Colocated: trainer and rollout engine time-slice
one GPU — before training, generation pauses (in-flight requests keep partial outputs) and the
engine's KV cache is released; before rollout, the trainer's gradient buffer is released and the
KV cache re-acquired.  Memory moves through the tagged VMM allocator when the two live in
different processes, or through plain buffer release when they share a process.  Disaggregated:
nothing is released, only generation is paused around the weight push.
"""

from __future__ import annotations

from typing import Any


class StageManager:
    def __init__(self, train_engine: Any, rollout_worker: Any) -> None:
        self.train, self.worker = train_engine, rollout_worker
        self.stage = "init"

    def switch_to_rollout(self) -> None:
        raise NotImplementedError

    def switch_to_train(self) -> None:
        raise NotImplementedError

    def switch_to_weight_sync(self) -> None:
        raise NotImplementedError


class ColocatedStageManager(StageManager):
    def switch_to_train(self) -> None:
        self.worker.pause_generation()
        if getattr(self.train, "optim", None) is not None:
            self.train.optim.alloc_grads()
        self.stage = "train"

    def switch_to_weight_sync(self) -> None:
        self.stage = "sync"

    def switch_to_rollout(self) -> None:
        if getattr(self.train, "optim", None) is not None:
            self.train.optim.release_grads()
        self.worker.engine.reset_prefix_cache()
        self.worker.resume_generation()
        self.stage = "rollout"


class DisaggregatedStageManager(StageManager):
    def switch_to_train(self) -> None:
        self.stage = "train"

    def switch_to_weight_sync(self) -> None:
        self.worker.pause_generation()
        self.stage = "sync"

    def switch_to_rollout(self) -> None:
        self.worker.engine.reset_prefix_cache()
        self.worker.resume_generation()
        self.stage = "rollout"

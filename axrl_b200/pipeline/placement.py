"""GPU placement arithmetic for the pipeline roles.

Reference: ``get_worker_placement`` / ``initialize_pipeline_workers`` (``axrl/pipeline/utils.py:242-348``)
over Ray placement groups (``axrl/ray/resource_group.py``).  Here every GPU runs one process
(``torch.distributed``); placement decides which global ranks hold which role:

* colocated: trainer and rollout engines share every GPU (the trainer's DP x TP x PP x CP grid
  covers all ranks; engines of ``rollout_tp`` consecutive ranks);
* disaggregated: the first ``trainer_gpus`` ranks train, the rest serve rollout engines;
* a value model (PPO) shares the actor's ranks.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Placement:
    world: int
    trainer_ranks: list[int]
    rollout_engines: list[list[int]]
    value_ranks: list[int] = field(default_factory=list)
    colocated: bool = True

    def roles_of(self, rank: int) -> list[str]:
        roles = []
        if rank in self.trainer_ranks:
            roles.append("trainer")
        if any(rank in e for e in self.rollout_engines):
            roles.append("rollout")
        if rank in self.value_ranks:
            roles.append("value")
        return roles


def get_worker_placement(world: int, *, colocated: bool = True, trainer_gpus: int | None = None, rollout_tp: int = 1,
                         trainer_model_parallel: int = 1, with_value: bool = False) -> Placement:
    """``trainer_model_parallel`` = TP x PP x CP of the trainer (must divide its GPU count)."""
    assert world >= 1 and rollout_tp >= 1
    if colocated:
        trainer = list(range(world))
        rollout_pool = list(range(world))
    else:
        assert trainer_gpus is not None and 0 < trainer_gpus < world, "disaggregated placement needs 0 < trainer_gpus < world"
        trainer = list(range(trainer_gpus))
        rollout_pool = list(range(trainer_gpus, world))
    assert len(trainer) % trainer_model_parallel == 0, "trainer GPUs must be a multiple of TP x PP x CP"
    assert len(rollout_pool) % rollout_tp == 0, "rollout GPUs must be a multiple of the rollout TP size"
    engines = [rollout_pool[i:i + rollout_tp] for i in range(0, len(rollout_pool), rollout_tp)]
    return Placement(world=world, trainer_ranks=trainer, rollout_engines=engines, value_ranks=list(trainer) if with_value else [],
                     colocated=colocated)

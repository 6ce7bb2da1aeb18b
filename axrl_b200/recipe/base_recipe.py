"""User hook surface of an RL recipe (reference ``axrl/recipe/base_recipe.py:18-110``).

A recipe owns dataset registration, optional driver-side services and the per-conversation
``run_rollout`` coroutine.  Rollout loops call ``run_rollout(conversation, runtime)`` where
``runtime`` carries the rollout worker (router over engines), actor-local processors and
shared workers.
"""

from __future__ import annotations

from typing import Any, Mapping, Sequence


class BaseRecipe:
    def __init__(self, config: Any) -> None:
        self.config = config

    async def register_datasets(self) -> None:
        """Register recipe dataset classes before the controller loads datasets."""

    def prepare_dataset(self, dataset: Any, config: Any) -> None:
        _ = dataset, config

    def validate_dataset(self, dataset: Any, config: Any) -> None:
        _ = dataset, config

    async def start_services(self) -> dict[str, Any]:
        return {}

    async def stop_services(self, services: Mapping[str, Any]) -> None:
        _ = services

    async def shutdown(self) -> None:
        pass

    def get_train_dataset_configs(self) -> Sequence[Any] | None:
        return None

    def get_test_dataset_configs(self) -> Sequence[Any] | None:
        return None

    def get_test_datasets(self) -> list[tuple[str, Any]]:
        """(name, dataset) pairs evaluated by ``eval_only`` and the periodic evals."""
        return []

    def build_sft_samples(self, dataset: Any) -> list:
        """SFT samples (prompt + target tokens, loss on the target) of ``dataset`` for ``sft_train``."""
        raise NotImplementedError(f"{self.__class__.__name__} does not provide SFT samples")

    async def run_rollout(self, conversation: Any, runtime: Any) -> Any:
        raise NotImplementedError(f"{self.__class__.__name__}.run_rollout() must be implemented")

    def initialize_local_processors(self, worker_id: str) -> Mapping[str, Any]:
        _ = worker_id
        return {}

    def initialize_shared_workers(self, services: Mapping[str, Any]) -> dict[str, Any]:
        _ = services
        return {}

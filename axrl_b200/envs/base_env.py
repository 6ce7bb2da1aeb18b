"""Gym-like environment interface (reference ``axrl/envs/base_env.py:8-14``)."""

from __future__ import annotations

import copy
from typing import Any

from axrl_b200.data.conversation import Conversation


class BaseEnv:
    def __init__(self, conv: Conversation) -> None:
        self.conv = copy.deepcopy(conv)

    async def step(self, action: Any) -> tuple[Conversation, float, bool, Any, Any]:
        """Returns (observation conversation, reward, done, trace, metric)."""
        raise NotImplementedError

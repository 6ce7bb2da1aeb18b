"""Agent interface (reference ``axrl/agent/base_agent.py:9-15``)."""

from __future__ import annotations

from typing import Any

from axrl_b200.data.conversation import Conversation


class BaseAgent:
    async def act(self, conversation: Conversation, config: Any) -> Any:
        raise NotImplementedError

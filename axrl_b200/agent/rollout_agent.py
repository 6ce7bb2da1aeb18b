"""Agent that asks the rollout engine for the next assistant turn (reference ``axrl/agent/rollout_agent.py:17-45``)."""

from __future__ import annotations

from typing import Any

import numpy as np

from axrl_b200.agent.base_agent import BaseAgent
from axrl_b200.data.conversation import Conversation, GenerationInput


class RolloutAgent(BaseAgent):
    def __init__(self, rollout_worker: Any, sampling_config: Any = None) -> None:
        self.worker = rollout_worker
        self.sampling_config = sampling_config

    async def act(self, conversation: Conversation, config: Any = None) -> Any:
        gs = conversation.gen_state
        assert gs.input_ids is not None, "conversation must be tokenised before act()"
        inp = GenerationInput(session_id=gs.session_id or conversation.conversation_id, input_ids=np.asarray(gs.input_ids),
                              sampling_config=config or gs.sampling_config or self.sampling_config, tools=gs.tools,
                              tool_choice=gs.tool_choice, tool_call_parser=gs.tool_call_parser, capture_routing=gs.capture_routing,
                              routed_expert_start_index=gs.captured_routing_rows)
        return await self.worker.generate(inp)

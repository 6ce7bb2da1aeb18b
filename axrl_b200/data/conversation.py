"""Conversation and generation records exchanged between envs, agents and the rollout engine.

Field names follow reference ``axrl/data/conversation.py:13-167``,
``axrl/data/generation.py:13-91``, ``axrl/data/rollout_result.py:16-27`` and
``axrl/data/event_timing.py:7-67`` so recipes can be moved over unchanged.
"""

from __future__ import annotations

import copy
import time
from dataclasses import dataclass, field
from typing import Any, Literal

import numpy as np

from axrl_b200.configs import SamplingConfig


@dataclass
class MessagePart:
    type: Literal["text", "image"]
    text: str | None = None
    image: str | None = None
    extra: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict:
        d: dict = {"type": self.type}
        if self.text is not None:
            d["text"] = self.text
        if self.image is not None:
            d["image"] = self.image
        if self.extra:
            d["extra"] = dict(self.extra)
        return d

    @staticmethod
    def from_dict(d: dict) -> "MessagePart":
        return MessagePart(type=d["type"], text=d.get("text"), image=d.get("image"), extra=dict(d.get("extra", {})))


@dataclass
class ToolCall:
    id: str
    index: int
    name: str
    arguments: str  # JSON string

    def to_dict(self) -> dict[str, Any]:
        return {"id": self.id, "type": "function", "function": {"name": self.name, "arguments": self.arguments}}

    @staticmethod
    def from_dict(d: dict[str, Any], index: int = 0) -> "ToolCall":
        return ToolCall(id=d["id"], index=index, name=d["function"]["name"], arguments=d["function"]["arguments"])


@dataclass
class Message:
    role: Literal["user", "assistant", "system", "tool"]
    content: str | list[MessagePart]
    tool_calls: list[ToolCall] | None = None
    tool_call_id: str | None = None
    extra: dict[str, Any] = field(default_factory=dict)

    def text(self) -> str:
        if isinstance(self.content, str):
            return self.content
        return "".join(p.text or "" for p in self.content)

    def to_dict(self) -> dict:
        d: dict = {"role": self.role, "content": self.content if isinstance(self.content, str) else [p.to_dict() for p in self.content]}
        if self.tool_calls:
            d["tool_calls"] = [t.to_dict() for t in self.tool_calls]
        if self.tool_call_id is not None:
            d["tool_call_id"] = self.tool_call_id
        if self.extra:
            d["extra"] = dict(self.extra)
        return d

    @staticmethod
    def from_dict(d: dict) -> "Message":
        c = d["content"]
        content = c if isinstance(c, str) else [MessagePart.from_dict(p) for p in c]
        tcs = [ToolCall.from_dict(t, i) for i, t in enumerate(d["tool_calls"])] if d.get("tool_calls") else None
        return Message(role=d["role"], content=content, tool_calls=tcs, tool_call_id=d.get("tool_call_id"), extra=dict(d.get("extra", {})))


@dataclass
class GenerationState:
    session_id: str | None = None
    input_ids: np.ndarray | None = None
    sampling_config: SamplingConfig | None = None
    tools: list[dict[str, Any]] | None = None
    tool_choice: str | dict[str, Any] | None = None
    tool_call_parser: str | None = None
    capture_routing: bool = False
    captured_routing_rows: int = 0


@dataclass
class Conversation:
    messages: list[Message] = field(default_factory=list)
    conversation_id: str = ""
    extra: dict[str, Any] = field(default_factory=dict)
    source: str = ""
    gen_state: GenerationState = field(default_factory=GenerationState)

    def add_message(self, message: Message) -> None:
        self.messages.append(message)

    def deep_copy(self) -> "Conversation":
        return copy.deepcopy(self)

    def to_dict(self) -> dict:
        return {"messages": [m.to_dict() for m in self.messages], "conversation_id": self.conversation_id, "extra": dict(self.extra),
                "source": self.source}

    @staticmethod
    def from_dict(d: dict) -> "Conversation":
        return Conversation(messages=[Message.from_dict(m) for m in d["messages"]], conversation_id=d.get("conversation_id", ""),
                            extra=dict(d.get("extra", {})), source=d.get("source", ""))


@dataclass
class EventTiming:
    """Four stamps of one request's trip: scheduled -> worker received -> worker returned -> driver received."""

    scheduled: float | None = None
    worker_received: float | None = None
    worker_returned: float | None = None
    driver_received: float | None = None

    def stamp(self, name: str) -> None:
        setattr(self, name, time.time())

    def overhead_seconds(self) -> float | None:
        if None in (self.scheduled, self.worker_received, self.worker_returned, self.driver_received):
            return None
        return (self.worker_received - self.scheduled) + (self.driver_received - self.worker_returned)


@dataclass
class GenerationInput:
    session_id: str
    input_ids: np.ndarray
    sampling_config: SamplingConfig | None = None
    lora_path: str | None = None
    tools: list[dict[str, Any]] | None = None
    tool_choice: str | dict[str, Any] | None = None
    tool_call_parser: str | None = None
    capture_input_logprobs: bool = False
    input_logprob_start_index: int = 0
    capture_routing: bool = False
    routed_expert_start_index: int = 0
    event_timing: EventTiming = field(default_factory=EventTiming)

    def __post_init__(self) -> None:
        self.input_ids = np.asarray(self.input_ids, dtype=np.int32)
        assert self.input_logprob_start_index >= 0


@dataclass
class GenerationOutput:
    session_id: str
    output_ids: np.ndarray
    output_logprobs: np.ndarray
    output_text: str
    output_text_with_special_tokens: str
    cached_tokens: int
    finish_reason: str
    e2e_elapsed_seconds: float
    stop_reason: int | str | None
    retry: int
    assistant_boundary_token_id: int | None = None
    tool_calls: list[ToolCall] | None = None
    input_logprobs: np.ndarray | None = None
    input_logprob_token_ids: np.ndarray | None = None
    input_logprob_start_index: int | None = None
    routing_handle: Any = None
    event_timing: EventTiming = field(default_factory=EventTiming)

    def __post_init__(self) -> None:
        self.output_ids = np.asarray(self.output_ids, dtype=np.int32)
        self.output_logprobs = np.asarray(self.output_logprobs, dtype=np.float32)


@dataclass
class RolloutResult:
    conversation: Conversation
    trace: Any  # RolloutTrace | None
    metric: Any  # ResponseMetric
    packed_samples: Any = None
    packed_samples_ref: Any = None
    trainable_token_count: int | None = None
    routing_handles: list | None = None
    reward: float | None = None
    reward_baseline: float | None = None
    scalar_advantage: float | None = None

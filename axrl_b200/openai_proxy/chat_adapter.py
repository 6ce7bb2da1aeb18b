"""Chat adapter: OpenAI chat request -> token ids -> generation -> OpenAI chat response.

Reference: ``OpenAIChatAdapter`` (``axrl/openai_proxy/chat_adapter.py:81-538``): render the
conversation with the model's chat template, run generation through the rollout worker, parse
tool calls from the completion, and build the ``chat.completion`` JSON with usage counts.
Tool calls use the Hermes ``<tool_call>{json}</tool_call>`` convention of Qwen models.
"""

from __future__ import annotations

import json
import re
import time
import uuid
from typing import Any, Callable

import numpy as np

from axrl_b200.data.conversation import GenerationInput, ToolCall

_TOOL_RE = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


def parse_tool_calls(text: str) -> tuple[str, list[ToolCall]]:
    calls = []
    for i, m in enumerate(_TOOL_RE.finditer(text)):
        try:
            obj = json.loads(m.group(1))
        except json.JSONDecodeError:
            continue
        calls.append(ToolCall(id=f"call_{uuid.uuid4().hex[:12]}", index=i, name=str(obj.get("name", "")),
                              arguments=json.dumps(obj.get("arguments", {}))))
    return (_TOOL_RE.sub("", text).strip() if calls else text), calls


class OpenAIChatAdapter:
    def __init__(self, render: Callable[[list[dict], list[dict] | None], list[int]], decode: Callable[[list[int]], str],
                 model_name: str = "axrl-policy") -> None:
        """``render(messages, tools)`` applies the chat template and returns prompt token ids;
        ``decode(ids)`` detokenises the completion."""
        self.render, self.decode, self.model_name = render, decode, model_name

    def convert_request(self, body: dict[str, Any], session_id: str, sampling: Any = None) -> GenerationInput:
        ids = self.render(body.get("messages", []), body.get("tools"))
        return GenerationInput(session_id=session_id, input_ids=np.asarray(ids, np.int32), sampling_config=sampling,
                               tools=body.get("tools"), tool_choice=body.get("tool_choice"))

    def build_response(self, out: Any, prompt_tokens: int) -> dict[str, Any]:
        text = out.output_text or self.decode(out.output_ids.tolist())
        content, calls = parse_tool_calls(text)
        msg: dict[str, Any] = {"role": "assistant", "content": content}
        if calls:
            msg["tool_calls"] = [c.to_dict() for c in calls]
        finish = "tool_calls" if calls else ("length" if out.finish_reason == "length" else "stop")
        n = len(out.output_ids)
        return {"id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion", "created": int(time.time()), "model": self.model_name,
                "choices": [{"index": 0, "message": msg, "finish_reason": finish}],
                "usage": {"prompt_tokens": prompt_tokens, "completion_tokens": n, "total_tokens": prompt_tokens + n}}

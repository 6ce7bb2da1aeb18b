"""Chat adapter: OpenAI chat request -> token ids -> generation -> OpenAI chat response.

Reference: ``OpenAIChatAdapter`` (``axrl/openai_proxy/chat_adapter.py:81-538``).

* **Rendering**: the conversation goes through the model's chat template (``tokenizer`` or a
  ``render(messages, tools)`` callable); assistant tool-call arguments given as JSON strings are
  decoded for the template, tools are passed unless ``tool_choice == "none"``, and
  ``chat_template_kwargs`` reach the template.
* **Validation**: requests the rollout cannot honour are rejected with ``ValueError`` before any
  generation (``stream``, ``n != 1``, logprobs, response formats, logit bias, seeds, stop-token
  and grammar fields, multimodal content, ``tool_choice`` without tools).  Sampling fields are
  ignored on purpose: the trainer's sampling config governs every rollout.
* **Parsers** (``parsers.py``): the tool-call and reasoning parsers are resolved once from the
  configuration — ``None`` off, ``"auto"`` detected from the chat template, or a named parser.
* **Response**: reasoning text is split off into ``reasoning_content`` (unless the request sets
  ``separate_reasoning: false``), tool calls are parsed when the request carries tools, the finish
  reason becomes ``tool_calls`` when calls were found, and usage counts prompt and completion tokens.
"""

from __future__ import annotations

import json
import time
import uuid
from typing import Any, Callable

import numpy as np

from axrl_b200.data.conversation import GenerationInput, ToolCall
from axrl_b200.openai_proxy.parsers import (REASONING_PARSERS, TOOL_PARSERS, detect_reasoning, detect_tool_call_parser, parse_hermes,
                                            resolve_parser)

FINISH_REASONS = ("stop", "length", "tool_calls", "content_filter", "function_call", "abort")


def parse_tool_calls(text: str) -> tuple[str, list[ToolCall]]:
    """Hermes / Qwen ``<tool_call>{json}</tool_call>`` calls (the engine's native format)."""
    return parse_hermes(text)


def unsupported_request_fields(body: dict[str, Any]) -> list[str]:
    tools = body.get("tools")
    tc = body.get("tool_choice")
    checks = [
        (not body.get("messages"), "empty messages"),
        (isinstance(tc, str) and tc.lower() == "required" and not tools, "tool_choice=required without tools"),
        (tc is not None and not isinstance(tc, str) and not tools, "specific tool_choice without tools"),
        (bool(body.get("stream")), "stream=true"),
        (body.get("n", 1) not in (None, 1), "n != 1"),
        (bool(body.get("logprobs")) or bool(body.get("top_logprobs")), "logprobs/top_logprobs"),
        (body.get("response_format") is not None, "response_format"),
        (body.get("logit_bias") is not None, "logit_bias"),
        (body.get("seed") is not None, "seed"),
        (body.get("stop_token_ids") is not None, "stop_token_ids"),
        (body.get("stop_regex") is not None, "stop_regex"),
        (body.get("regex") is not None, "regex"),
        (body.get("ebnf") is not None, "ebnf"),
        (bool(body.get("min_tokens")), "min_tokens"),
        (bool(body.get("ignore_eos")), "ignore_eos"),
        (bool(body.get("return_hidden_states")), "return_hidden_states"),
        (isinstance(body.get("lora_path"), list), "batched lora_path"),
    ]
    for m in body.get("messages") or []:
        c = m.get("content") if isinstance(m, dict) else None
        if isinstance(c, list) and any(isinstance(p, dict) and p.get("type", "text") != "text" for p in c):
            checks.append((True, "multimodal content"))
            break
    return [name for bad, name in checks if bad]


def _template_messages(messages: list[dict]) -> list[dict]:
    out = []
    for m in messages:
        d = dict(m)
        c = d.get("content")
        if c is None:
            d["content"] = ""
        elif isinstance(c, list):  # text parts -> one string
            d["content"] = "".join(p.get("text", "") for p in c if isinstance(p, dict))
        if d.get("role") == "assistant" and isinstance(d.get("tool_calls"), list):
            calls = []
            for tc in d["tool_calls"]:
                tc = json.loads(json.dumps(tc))
                fn = tc.get("function")
                if isinstance(fn, dict) and isinstance(fn.get("arguments"), str):
                    try:
                        fn["arguments"] = json.loads(fn["arguments"])
                    except json.JSONDecodeError:
                        pass
                calls.append(tc)
            d["tool_calls"] = calls
        out.append(d)
    return out


class OpenAIChatAdapter:
    def __init__(self, render: Callable[..., list[int]] | None = None, decode: Callable[[list[int]], str] | None = None,
                 model_name: str = "axrl-policy", *, tokenizer: Any = None, chat_template: str | None = None,
                 tool_call_parser: str | None = "auto", reasoning_parser: str | None = None) -> None:
        """Render with ``tokenizer`` (an HF tokenizer or :class:`ChatTokenizer`) or with
        ``render(messages, tools[, **template_kwargs])``; decode with ``decode(ids)`` or the tokenizer."""
        self.tok = tokenizer
        self._render = render
        self._decode = decode
        self.model_name = model_name
        inner = getattr(tokenizer, "tok", tokenizer)
        self.chat_template = chat_template if chat_template is not None else getattr(inner, "chat_template", None)
        tmpl = self.chat_template
        # no template known (a render callback): the engine's models use the Qwen / Hermes format
        self.tool_parser = resolve_parser(tool_call_parser, "tool-call parser",
                                          lambda: detect_tool_call_parser(tmpl) if tmpl else "qwen25", TOOL_PARSERS)
        detected, self.force_reasoning = detect_reasoning(tmpl)
        self.reasoning_parser = resolve_parser(reasoning_parser, "reasoning parser", lambda: detected, REASONING_PARSERS)

    # ------------------------------------------------------------------ request side
    def render(self, messages: list[dict], tools: list[dict] | None, template_kwargs: dict | None = None) -> list[int]:
        msgs = _template_messages(messages)
        kw = dict(template_kwargs or {})
        if self._render is not None:
            return list(self._render(msgs, tools, **kw) if kw else self._render(msgs, tools))
        inner = getattr(self.tok, "tok", self.tok)
        out = inner.apply_chat_template(msgs, tools=tools, add_generation_prompt=True, tokenize=True, **kw)
        return list(out["input_ids"] if isinstance(out, dict) else out)

    def decode(self, ids: list[int]) -> str:
        if self._decode is not None:
            return self._decode(ids)
        return self.tok.decode(ids, skip_special_tokens=False) if self.tok is not None else ""

    def convert_request(self, body: dict[str, Any], session_id: str, sampling: Any = None) -> GenerationInput:
        bad = unsupported_request_fields(body)
        if bad:
            raise ValueError(f"OpenAI chat request fields not supported by the rollout: {', '.join(bad)}")
        tools = body.get("tools")
        tmpl_tools = None if (not tools or body.get("tool_choice") == "none") else tools
        ids = self.render(body.get("messages", []), tmpl_tools, body.get("chat_template_kwargs"))
        return GenerationInput(session_id=session_id, input_ids=np.asarray(ids, np.int32), sampling_config=sampling, tools=tools,
                               tool_choice=body.get("tool_choice"), tool_call_parser=self.tool_parser if tools else None)

    # ------------------------------------------------------------------ response side
    def split_reasoning(self, text: str, request: dict | None = None) -> tuple[str, str | None]:
        if not self.reasoning_parser or (request or {}).get("separate_reasoning", True) is False:
            return text, None
        kwargs = ((request or {}).get("chat_template_kwargs") or {})
        force = self.force_reasoning or bool(kwargs.get("enable_thinking") and REASONING_PARSERS[self.reasoning_parser].force)
        reasoning, normal = REASONING_PARSERS[self.reasoning_parser].parse(text, force)
        return normal, reasoning

    def build_response(self, out: Any, prompt_tokens: int, request: dict | None = None) -> dict[str, Any]:
        text = out.output_text or self.decode(out.output_ids.tolist())
        text, reasoning = self.split_reasoning(text, request)
        calls: list[ToolCall] = []
        has_tools = request is None or bool(request.get("tools"))
        if self.tool_parser and has_tools and (request or {}).get("tool_choice") != "none":
            text, calls = TOOL_PARSERS[self.tool_parser](text)
        msg: dict[str, Any] = {"role": "assistant", "content": text or None}
        if reasoning:
            msg["reasoning_content"] = reasoning
        if calls:
            msg["tool_calls"] = [c.to_dict() for c in calls]
        finish = out.finish_reason if out.finish_reason in FINISH_REASONS else "stop"
        if calls and finish == "stop":
            finish = "tool_calls"
        n = len(out.output_ids)
        return {"id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion", "created": int(time.time()),
                "model": (request or {}).get("model") or self.model_name,
                "choices": [{"index": 0, "message": msg, "finish_reason": finish,
                             "matched_stop": None if finish == "tool_calls" else getattr(out, "stop_reason", None)}],
                "usage": {"prompt_tokens": prompt_tokens, "completion_tokens": n, "total_tokens": prompt_tokens + n}}

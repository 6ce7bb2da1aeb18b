"""Tool-call and reasoning parsers for model completions, with chat-template auto-detection.

The reference resolves these by name from SGLang's registries (``axrl/openai_proxy/chat_adapter.py:
40-48, 184-251``): ``None`` disables a parser, ``"auto"`` detects it from the chat template, any
other name must be a known parser.  This module is the engine-independent equivalent: the parser
names are the ones SGLang users write in configs, each parser turns completion text into
``(normal_text, tool_calls)`` or ``(reasoning_text, normal_text)``, and detection reads the
markers a model family's chat template emits.

Tool-call formats:

* ``qwen25`` / ``qwen`` / ``hermes``: ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``
* ``qwen3_coder``: ``<tool_call><function=NAME><parameter=KEY>VALUE</parameter>...</function></tool_call>``
* ``glm45``: ``<tool_call>NAME\\n<arg_key>K</arg_key><arg_value>V</arg_value>...</tool_call>``
* ``mistral``: ``[TOOL_CALLS] [{"name": ..., "arguments": {...}}, ...]``
* ``llama3``: ``<|python_tag|>`` and/or bare ``{"name": ..., "parameters": {...}}`` objects, ``;``-separated
* ``deepseekv3``: ``<｜tool▁call▁begin｜>function<｜tool▁sep｜>NAME\\n```json\\n{...}\\n```<｜tool▁call▁end｜>``
* ``kimi_k2``: ``<|tool_call_begin|>functions.NAME:IDX<|tool_call_argument_begin|>{...}<|tool_call_end|>``
* ``pythonic``: ``[name(a=1, b="x"), other()]``

Reasoning formats: ``qwen3`` / ``glm45`` (``<think>...</think>``), ``deepseek-r1`` / ``step3`` (the
same tags, but the template opens the block, so text before ``</think>`` is reasoning even without an
opening tag), ``kimi`` (``◁think▷...◁/think▷``).
"""

from __future__ import annotations

import ast
import json
import re
import uuid
from typing import Callable

from axrl_b200.data.conversation import ToolCall


def _call(i: int, name: str, args: object) -> ToolCall:
    a = args if isinstance(args, str) else json.dumps(args if args is not None else {}, ensure_ascii=False)
    return ToolCall(id=f"call_{uuid.uuid4().hex[:24]}", index=i, name=str(name), arguments=a)


def _scalar(v: str) -> object:
    """A parameter value written as text: JSON when it parses, else the stripped string."""
    s = v.strip()
    try:
        return json.loads(s)
    except (json.JSONDecodeError, ValueError):
        return s


# ------------------------------------------------------------------------------- tool-call parsers
_HERMES = re.compile(r"<tool_call>\s*(.*?)\s*</tool_call>", re.S)


def parse_hermes(text: str) -> tuple[str, list[ToolCall]]:
    calls = []
    for m in _HERMES.finditer(text):
        try:
            obj = json.loads(m.group(1))
        except json.JSONDecodeError:
            continue
        if isinstance(obj, dict) and "name" in obj:
            calls.append(_call(len(calls), obj["name"], obj.get("arguments", obj.get("parameters", {}))))
    return (_HERMES.sub("", text).strip() if calls else text), calls


_XML_FN = re.compile(r"<function=([^>\s]+)>(.*?)</function>", re.S)
_XML_PARAM = re.compile(r"<parameter=([^>\s]+)>(.*?)</parameter>", re.S)


def parse_qwen3_coder(text: str) -> tuple[str, list[ToolCall]]:
    calls = []
    for block in _HERMES.finditer(text):
        for fn in _XML_FN.finditer(block.group(1)):
            args = {k: _scalar(v) for k, v in _XML_PARAM.findall(fn.group(2))}
            calls.append(_call(len(calls), fn.group(1), args))
    return (_HERMES.sub("", text).strip() if calls else text), calls


_GLM_ARG = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)


def parse_glm45(text: str) -> tuple[str, list[ToolCall]]:
    calls = []
    for block in _HERMES.finditer(text):
        body = block.group(1)
        name = body.split("<arg_key>", 1)[0].strip().splitlines()[0].strip() if body.strip() else ""
        if not name:
            continue
        calls.append(_call(len(calls), name, {k.strip(): _scalar(v) for k, v in _GLM_ARG.findall(body)}))
    return (_HERMES.sub("", text).strip() if calls else text), calls


def _json_prefix(s: str) -> tuple[object, int] | None:
    try:
        return json.JSONDecoder().raw_decode(s)
    except json.JSONDecodeError:
        return None


def parse_mistral(text: str) -> tuple[str, list[ToolCall]]:
    i = text.find("[TOOL_CALLS]")
    if i < 0:
        return text, []
    rest = text[i + len("[TOOL_CALLS]"):].lstrip()
    got = _json_prefix(rest)
    if got is None:
        return text, []
    objs = got[0] if isinstance(got[0], list) else [got[0]]
    calls = [_call(k, o["name"], o.get("arguments", {})) for k, o in enumerate(objs) if isinstance(o, dict) and "name" in o]
    return (text[:i].strip() if calls else text), calls


def parse_llama3(text: str) -> tuple[str, list[ToolCall]]:
    body = text.split("<|python_tag|>", 1)
    head, tail = (body[0], body[1]) if len(body) == 2 else ("", body[0])
    calls, pos = [], 0
    tail = tail.strip()
    while pos < len(tail):
        got = _json_prefix(tail[pos:])
        if got is None or not isinstance(got[0], dict) or "name" not in got[0]:
            break
        calls.append(_call(len(calls), got[0]["name"], got[0].get("parameters", got[0].get("arguments", {}))))
        pos += got[1]
        while pos < len(tail) and tail[pos] in "; \n\t":
            pos += 1
    if not calls:
        return text, []
    return (head + tail[pos:]).strip(), calls


_DSV3 = re.compile(r"<｜tool▁call▁begin｜>(\w+)<｜tool▁sep｜>([^\n]+)\n```json\n(.*?)\n```<｜tool▁call▁end｜>", re.S)


def parse_deepseekv3(text: str) -> tuple[str, list[ToolCall]]:
    calls = [_call(i, m.group(2).strip(), _scalar(m.group(3))) for i, m in enumerate(_DSV3.finditer(text))]
    if not calls:
        return text, []
    return text.split("<｜tool▁calls▁begin｜>", 1)[0].strip(), calls


_KIMI = re.compile(r"<\|tool_call_begin\|>\s*([^<]+?)\s*<\|tool_call_argument_begin\|>(.*?)<\|tool_call_end\|>", re.S)


def parse_kimi_k2(text: str) -> tuple[str, list[ToolCall]]:
    calls = []
    for m in _KIMI.finditer(text):
        ident = m.group(1)  # functions.NAME:IDX
        name = ident.split(".", 1)[-1].rsplit(":", 1)[0]
        calls.append(_call(len(calls), name, _scalar(m.group(2))))
    if not calls:
        return text, []
    return text.split("<|tool_calls_section_begin|>", 1)[0].strip(), calls


def parse_pythonic(text: str) -> tuple[str, list[ToolCall]]:
    m = re.search(r"\[\s*[A-Za-z_][\w.]*\(.*\)\s*\]", text, re.S)
    if not m:
        return text, []
    try:
        tree = ast.parse(m.group(0), mode="eval")
    except SyntaxError:
        return text, []
    if not isinstance(tree.body, ast.List):
        return text, []
    calls = []
    for el in tree.body.elts:
        if not isinstance(el, ast.Call):
            return text, []
        try:
            args = {kw.arg: ast.literal_eval(kw.value) for kw in el.keywords}
        except ValueError:
            return text, []
        calls.append(_call(len(calls), ast.unparse(el.func), args))
    return (text[:m.start()] + text[m.end():]).strip(), calls


TOOL_PARSERS: dict[str, Callable[[str], tuple[str, list[ToolCall]]]] = {
    "qwen25": parse_hermes, "qwen": parse_hermes, "hermes": parse_hermes, "qwen3_coder": parse_qwen3_coder, "glm45": parse_glm45,
    "glm47": parse_glm45, "mistral": parse_mistral, "llama3": parse_llama3, "deepseekv3": parse_deepseekv3, "kimi_k2": parse_kimi_k2,
    "pythonic": parse_pythonic,
}


# ------------------------------------------------------------------------------- reasoning parsers
class ThinkParser:
    """Splits ``<open>reasoning<close>answer``; ``force`` treats text before ``<close>`` as reasoning
    when the template already opened the block (the completion then has no opening tag)."""

    def __init__(self, open_tag: str = "<think>", close_tag: str = "</think>", force: bool = False) -> None:
        self.open, self.close, self.force = open_tag, close_tag, force

    def parse(self, text: str, force: bool | None = None) -> tuple[str | None, str]:
        force = self.force if force is None else force
        s = text
        i = s.find(self.open)
        if i >= 0:
            pre, s = s[:i], s[i + len(self.open):]
        elif not force:
            return None, text
        else:
            pre = ""
        j = s.find(self.close)
        if j < 0:  # unterminated block: everything after the tag is reasoning
            return s.strip() or None, pre.strip()
        return s[:j].strip() or None, (pre + s[j + len(self.close):]).strip()


REASONING_PARSERS: dict[str, ThinkParser] = {
    "qwen3": ThinkParser(), "qwen3-thinking": ThinkParser(force=True), "glm45": ThinkParser(), "deepseek-r1": ThinkParser(force=True),
    "deepseek-v3": ThinkParser(), "step3": ThinkParser(force=True), "kimi": ThinkParser("◁think▷", "◁/think▷"),
    "minimax": ThinkParser(force=True),
}


# ------------------------------------------------------------------------------- detection
def detect_tool_call_parser(template: str | None) -> str | None:
    """Tool-call format a chat template renders (its tool-call markers)."""
    t = template or ""
    if "<tool_call>" in t and "<function=" in t:
        return "qwen3_coder"
    if "<tool_call>" in t and "<arg_key>" in t:
        return "glm45"
    if "<tool_call>" in t:
        return "qwen25"
    if "[TOOL_CALLS]" in t:
        return "mistral"
    if "<｜tool▁calls▁begin｜>" in t:
        return "deepseekv3"
    if "<|tool_calls_section_begin|>" in t or "<|tool_call_begin|>" in t:
        return "kimi_k2"
    if "<|python_tag|>" in t:
        return "llama3"
    return None


def detect_reasoning(template: str | None) -> tuple[str | None, bool]:
    """(reasoning parser, force_reasoning) for a chat template: a template whose generation prompt
    already opens the thinking block forces reasoning."""
    t = template or ""
    if "◁think▷" in t:
        return "kimi", False
    if "<think>" not in t:
        return None, False
    forced = bool(re.search(r"add_generation_prompt[^%]*%\}[^{]*assistant[^{]*<think>", t, re.S)) or "<|Assistant|><think>" in t \
        or "'<think>\\n'" in t.split("add_generation_prompt")[-1]
    return ("deepseek-r1" if forced else "qwen3"), forced


def resolve_parser(configured: str | None, label: str, auto: Callable[[], str | None], registry: dict) -> str | None:
    """``None`` / empty: disabled; ``"auto"``: detected (None when nothing matches); else the name
    must be registered."""
    if configured is None or not configured.strip():
        return None
    name = configured.strip().lower()
    if name == "auto":
        return auto()
    if name not in registry:
        raise ValueError(f"unsupported {label}: {configured!r} (known: {sorted(registry)})")
    return name

"""OpenAI proxy: real HTTP on localhost through the registry, 404 / 504 / 499 paths, auth, tool-call parsing."""

import asyncio

import httpx
import numpy as np

from axrl_b200.data.conversation import GenerationOutput
from axrl_b200.openai_proxy.chat_adapter import OpenAIChatAdapter, parse_tool_calls
from axrl_b200.openai_proxy.server import OpenAIProxyServer, OpenAIProxySessionRegistry


def test_parse_tool_calls():
    text, calls = parse_tool_calls('ok <tool_call>{"name": "search", "arguments": {"q": "x"}}</tool_call>')
    assert text == "ok" and calls[0].name == "search" and '"q"' in calls[0].arguments


def test_http_roundtrip_and_errors():
    async def go():
        reg = OpenAIProxySessionRegistry(request_timeout_seconds=1.0)
        srv = OpenAIProxyServer(reg, api_key="k")
        srv.start(asyncio.get_running_loop())
        await srv.wait_started()
        adapter = OpenAIChatAdapter(render=lambda msgs, tools: [1, 2, 3], decode=lambda ids: "hi")
        await reg.create_session("s1")

        async def env_side():
            req = await reg.wait_for_request("s1")
            inp = adapter.convert_request(req.body, "s1")
            out = GenerationOutput("s1", np.array([5, 6]), np.array([-0.1, -0.2]), "hello", "hello", 0, "stop", 0.0, None, 0)
            await reg.respond(req.request_id, adapter.build_response(out, len(inp.input_ids)))

        async with httpx.AsyncClient(timeout=5) as c:
            h = {"Authorization": "Bearer k"}
            env = asyncio.create_task(env_side())
            r = await c.post(srv.base_url("s1") + "/chat/completions", json={"messages": [{"role": "user", "content": "x"}]}, headers=h)
            await env
            assert r.status_code == 200 and r.json()["choices"][0]["message"]["content"] == "hello"
            assert r.json()["usage"] == {"prompt_tokens": 3, "completion_tokens": 2, "total_tokens": 5}
            assert (await c.post(srv.base_url("nope") + "/chat/completions", json={}, headers=h)).status_code == 404
            assert (await c.post(srv.base_url("s1") + "/chat/completions", json={})).status_code == 401
            assert (await c.post(srv.base_url("s1") + "/chat/completions", json={}, headers=h)).status_code == 504
            pending = asyncio.create_task(c.post(srv.base_url("s1") + "/chat/completions", json={}, headers=h))
            await asyncio.sleep(0.2)
            await reg.close_session("s1")
            assert (await pending).status_code == 499
        await srv.stop()

    asyncio.run(go())


def test_tool_call_parsers():
    from axrl_b200.openai_proxy.parsers import TOOL_PARSERS

    cases = {
        "qwen25": ('a <tool_call>{"name": "f", "arguments": {"x": 1}}</tool_call>', "a", "f", {"x": 1}),
        "qwen3_coder": ("b <tool_call><function=g><parameter=q>hi</parameter><parameter=n>3</parameter></function></tool_call>", "b", "g",
                        {"q": "hi", "n": 3}),
        "glm45": ("c <tool_call>h\n<arg_key>k</arg_key><arg_value>[1, 2]</arg_value></tool_call>", "c", "h", {"k": [1, 2]}),
        "mistral": ('d [TOOL_CALLS] [{"name": "m", "arguments": {"z": true}}]', "d", "m", {"z": True}),
        "llama3": ('<|python_tag|>{"name": "l", "parameters": {"u": "v"}}', "", "l", {"u": "v"}),
        "deepseekv3": ('e<｜tool▁calls▁begin｜><｜tool▁call▁begin｜>function<｜tool▁sep｜>ds\n```json\n{"a": 1}\n```<｜tool▁call▁end｜>'
                       '<｜tool▁calls▁end｜>', "e", "ds", {"a": 1}),
        "kimi_k2": ('f<|tool_calls_section_begin|><|tool_call_begin|>functions.kk:0<|tool_call_argument_begin|>{"b": 2}<|tool_call_end|>'
                    '<|tool_calls_section_end|>', "f", "kk", {"b": 2}),
        "pythonic": ('g [search(query="x", k=2)]', "g", "search", {"query": "x", "k": 2}),
    }
    import json

    for name, (text, rest, fn, args) in cases.items():
        normal, calls = TOOL_PARSERS[name](text)
        assert normal == rest, (name, normal)
        assert len(calls) == 1 and calls[0].name == fn and json.loads(calls[0].arguments) == args, name
        assert TOOL_PARSERS[name]("no calls here") == ("no calls here", [])


def test_reasoning_parsers_and_detection():
    import pytest

    from axrl_b200.openai_proxy.parsers import REASONING_PARSERS, detect_reasoning, detect_tool_call_parser, resolve_parser

    assert REASONING_PARSERS["qwen3"].parse("<think>plan</think>answer") == ("plan", "answer")
    assert REASONING_PARSERS["qwen3"].parse("just answer") == (None, "just answer")
    assert REASONING_PARSERS["deepseek-r1"].parse("plan</think>answer") == ("plan", "answer")
    assert REASONING_PARSERS["kimi"].parse("◁think▷p◁/think▷a") == ("p", "a")
    qwen3 = "{% for m in messages %}<|im_start|>{{ m.role }}{% endfor %}<tool_call>\n{{ tool }}</tool_call><think>"
    assert detect_tool_call_parser(qwen3) == "qwen25"
    assert detect_tool_call_parser("<tool_call><function=x>") == "qwen3_coder"
    assert detect_tool_call_parser("[TOOL_CALLS]") == "mistral"
    assert detect_tool_call_parser("plain") is None
    assert detect_reasoning(qwen3) == ("qwen3", False)
    assert detect_reasoning("{% if add_generation_prompt %}<|Assistant|><think>\n{% endif %}")[1] is True
    assert resolve_parser(None, "x", lambda: "q", {"q": 1}) is None
    assert resolve_parser("auto", "x", lambda: "q", {"q": 1}) == "q"
    with pytest.raises(ValueError):
        resolve_parser("nope", "x", lambda: None, {"q": 1})


def test_adapter_validation_reasoning_and_tool_response():
    import pytest

    adapter = OpenAIChatAdapter(render=lambda msgs, tools: [1, 2, 3] if tools is None else [1, 2, 3, 4], decode=lambda ids: "",
                                chat_template="<tool_call><think>", tool_call_parser="auto", reasoning_parser="auto")
    assert adapter.tool_parser == "qwen25" and adapter.reasoning_parser == "qwen3"
    with pytest.raises(ValueError, match="stream"):
        adapter.convert_request({"messages": [{"role": "user", "content": "x"}], "stream": True}, "s")
    with pytest.raises(ValueError, match="required"):
        adapter.convert_request({"messages": [{"role": "user", "content": "x"}], "tool_choice": "required"}, "s")
    tools = [{"type": "function", "function": {"name": "f", "parameters": {}}}]
    body = {"messages": [{"role": "user", "content": "x"}, {"role": "assistant", "content": None,
                                                           "tool_calls": [{"id": "1", "type": "function",
                                                                           "function": {"name": "f", "arguments": "{\"a\": 1}"}}]}],
            "tools": tools}
    inp = adapter.convert_request(body, "s")
    assert len(inp.input_ids) == 4 and inp.tool_call_parser == "qwen25"
    out = GenerationOutput("s", np.array([5, 6, 7]), np.zeros(3), '<think>hmm</think>sure <tool_call>{"name": "f", "arguments": {}}</tool_call>',
                           "", 0, "stop", 0.0, None, 0)
    r = adapter.build_response(out, 4, body)
    msg = r["choices"][0]["message"]
    assert msg["reasoning_content"] == "hmm" and msg["content"] == "sure" and msg["tool_calls"][0]["function"]["name"] == "f"
    assert r["choices"][0]["finish_reason"] == "tool_calls"
    r2 = adapter.build_response(out, 4, {**body, "separate_reasoning": False, "tool_choice": "none"})
    assert "reasoning_content" not in r2["choices"][0]["message"] and r2["choices"][0]["finish_reason"] == "stop"

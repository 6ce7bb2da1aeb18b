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

"""OpenAI-compatible proxy for black-box agent harnesses.

Reference: ``axrl/openai_proxy/server.py:71-478``.  An external agent (e.g. an OpenHands
process in a sandbox) posts ``/sessions/{session_id}/v1/chat/completions`` to one shared HTTP
server.  The session registry parks each HTTP request as a future and hands the raw request
body to the rollout environment that owns the session (``wait_for_request``); the environment
renders it to token ids, generates with the rollout engine, builds the OpenAI response and
resolves the future (``respond``).  Unknown / closed sessions answer 404, a request that waits
longer than the timeout answers 504, closing a session fails its pending requests with 499.
Optional bearer-token auth.
"""

from __future__ import annotations

import asyncio
import time
import uuid
from dataclasses import dataclass, field
from typing import Any


@dataclass
class OpenAIPendingRequest:
    session_id: str
    request_id: str
    body: dict[str, Any]
    headers: dict[str, str]
    created_at: float


@dataclass
class OpenAIProxyResponse:
    body: dict[str, Any]
    status_code: int = 200
    headers: dict[str, str] = field(default_factory=dict)


def _err(msg: str, kind: str, code: int) -> OpenAIProxyResponse:
    return OpenAIProxyResponse({"error": {"message": msg, "type": kind, "code": code}}, code)


class OpenAIProxySessionRegistry:
    def __init__(self, request_timeout_seconds: float = 600.0) -> None:
        self.timeout = request_timeout_seconds
        self._queues: dict[str, asyncio.Queue] = {}
        self._futures: dict[str, tuple[OpenAIPendingRequest, asyncio.Future]] = {}
        self._closed: set[str] = set()

    async def create_session(self, session_id: str) -> None:
        if session_id in self._queues:
            raise ValueError(f"session already exists: {session_id}")
        self._queues[session_id] = asyncio.Queue()
        self._closed.discard(session_id)

    async def close_session(self, session_id: str) -> None:
        self._closed.add(session_id)
        self._queues.pop(session_id, None)
        for rid, (req, _) in list(self._futures.items()):
            if req.session_id == session_id:
                await self.fail(rid, "session was closed", status_code=499)

    async def submit_chat_completion(self, *, session_id: str, body: dict[str, Any], headers: dict[str, str]) -> OpenAIProxyResponse:
        if session_id in self._closed:
            return _err(f"session is closed: {session_id}", "not_found", 404)
        q = self._queues.get(session_id)
        if q is None:
            return _err(f"unknown session: {session_id}", "not_found", 404)
        req = OpenAIPendingRequest(session_id, uuid.uuid4().hex, body, headers, time.time())
        fut = asyncio.get_running_loop().create_future()
        self._futures[req.request_id] = (req, fut)
        await q.put(req)
        try:
            return await asyncio.wait_for(fut, self.timeout)
        except asyncio.TimeoutError:
            self._futures.pop(req.request_id, None)
            return _err("timed out waiting for the rollout response", "timeout", 504)

    async def wait_for_request(self, session_id: str, *, timeout_seconds: float | None = None) -> OpenAIPendingRequest:
        q = self._queues.get(session_id)
        if q is None:
            raise KeyError(f"unknown session: {session_id}")
        while True:
            req = await (q.get() if timeout_seconds is None else asyncio.wait_for(q.get(), timeout_seconds))
            if req.request_id in self._futures:
                return req

    async def respond(self, request_id: str, body: dict[str, Any], *, status_code: int = 200, headers: dict[str, str] | None = None) -> None:
        item = self._futures.pop(request_id, None)
        if item is None or item[1].done():
            return
        item[1].set_result(OpenAIProxyResponse(body, status_code, headers or {}))

    async def fail(self, request_id: str, message: str, *, status_code: int = 500) -> None:
        await self.respond(request_id, {"error": {"message": message, "type": "openai_proxy_error", "code": status_code}}, status_code=status_code)


def create_app(registry: OpenAIProxySessionRegistry, api_key: str | None = None):  # noqa: ANN201
    """FastAPI app exposing the proxy routes."""
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse

    app = FastAPI()
    # Route signatures are resolved by FastAPI from annotations; with postponed annotations the
    # names must be visible in module globals.
    globals()["Request"] = Request

    def _auth(request: Request) -> JSONResponse | None:
        if api_key is None:
            return None
        if request.headers.get("authorization", "") != f"Bearer {api_key}":
            return JSONResponse({"error": {"message": "invalid api key", "type": "auth", "code": 401}}, status_code=401)
        return None

    @app.get("/health")
    async def health() -> dict:
        return {"ok": True}

    @app.post("/sessions/{session_id}/v1/chat/completions")
    async def chat(session_id: str, request: Request):  # noqa: ANN202
        bad = _auth(request)
        if bad is not None:
            return bad
        body = await request.json()
        resp = await registry.submit_chat_completion(session_id=session_id, body=body, headers=dict(request.headers))
        return JSONResponse(resp.body, status_code=resp.status_code, headers=resp.headers)

    @app.get("/sessions/{session_id}/v1/models")
    async def models(session_id: str) -> dict:
        return {"object": "list", "data": [{"id": "axrl-policy", "object": "model"}]}

    return app


class OpenAIProxyServer:
    """uvicorn server in a background thread; ``base_url(session)`` is what the harness is given."""

    def __init__(self, registry: OpenAIProxySessionRegistry, host: str = "127.0.0.1", port: int = 0, api_key: str | None = None) -> None:
        import socket

        self.registry, self.host, self.api_key = registry, host, api_key
        if port == 0:
            with socket.socket() as s:
                s.bind((host, 0))
                port = s.getsockname()[1]
        self.port = port
        self._server = None
        self._thread = None

    def base_url(self, session_id: str) -> str:
        return f"http://{self.host}:{self.port}/sessions/{session_id}/v1"

    def start(self, loop: asyncio.AbstractEventLoop) -> None:
        """Serve on ``loop`` (the loop that owns the registry's futures)."""
        import uvicorn

        cfg = uvicorn.Config(create_app(self.registry, self.api_key), host=self.host, port=self.port, log_level="warning", loop="asyncio")
        self._server = uvicorn.Server(cfg)
        self._task = loop.create_task(self._server.serve())

    async def wait_started(self, timeout: float = 10.0) -> None:
        t0 = time.time()
        while not (self._server and self._server.started):
            if time.time() - t0 > timeout:
                raise TimeoutError("proxy did not start")
            await asyncio.sleep(0.02)

    async def stop(self) -> None:
        if self._server is not None:
            self._server.should_exit = True
            await self._task

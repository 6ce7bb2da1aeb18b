"""HTTP router in front of several engine servers: least-loaded dispatch with session affinity
(bounded imbalance), health checks.

Reference: ``sglang_router`` launched by ``start_sglang_router`` (``axrl/utils/sglang_launch_utils.py:286``)
and the in-process ``InferenceRouter`` policy (``axrl/worker/infer_router.py``).

``python -m axrl_b200.serve.router --backends http://127.0.0.1:30000,http://127.0.0.1:30001 --port 30100``
"""

from __future__ import annotations

import argparse
from typing import Any


class _HttpBackend:
    def __init__(self, url: str) -> None:
        import httpx

        self.url = url.rstrip("/")
        self.http = httpx.AsyncClient(base_url=self.url, timeout=None)

    async def generate(self, body: dict) -> dict:
        r = await self.http.post("/generate", json=body)
        r.raise_for_status()
        return r.json()


class _Req:
    def __init__(self, body: dict) -> None:
        self.body = body
        self.session_id = str(body.get("rid")) if body.get("rid") is not None else None


def create_router_app(backends: list[str], max_imbalance: int = 16):  # noqa: ANN201
    from fastapi import FastAPI

    from axrl_b200.worker.infer_router import InferenceRouter

    class _Adapter:
        def __init__(self, be: _HttpBackend) -> None:
            self.be = be

        async def generate(self, req: _Req) -> Any:
            return await self.be.generate(req.body)

    router = InferenceRouter([_Adapter(_HttpBackend(u)) for u in backends], max_imbalance=max_imbalance)
    app = FastAPI()

    @app.post("/generate")
    async def generate(body: dict) -> dict:
        return await router.generate(_Req(body))

    @app.get("/health")
    async def health() -> dict:
        return {"ok": True, "backends": len(backends), "load": list(router.load)}

    return app


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--backends", required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30100)
    ap.add_argument("--max-imbalance", type=int, default=16)
    a = ap.parse_args(argv)
    import uvicorn

    uvicorn.run(create_router_app(a.backends.split(","), a.max_imbalance), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()

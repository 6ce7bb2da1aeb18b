"""Runner that executes commands in a remote sandbox service over HTTP.

Reference: ``E2BRunner`` (``axrl/runner/e2b_runner.py:40-269``), which drives E2B sandboxes
(create, run a command with a timeout, read output, kill).  This client speaks a small REST
protocol to a sandbox service at ``base_url``:

* ``POST /sandboxes`` ``{"template": ..., "timeout_s": ...}`` -> ``{"id": ...}``
* ``POST /sandboxes/{id}/exec`` ``{"command": ..., "cwd": ..., "timeout_s": ...}`` -> ``{"exit_code": int, "output": str}``
* ``DELETE /sandboxes/{id}``

An E2B (or any other) backend is adapted by a service implementing these three calls.
"""

from __future__ import annotations

import asyncio
from pathlib import Path

from axrl_b200.runner.base_runner import DEFAULT_TERMINATE_TIMEOUT_SECONDS, BaseRunner


class RemoteSandboxRunner(BaseRunner):
    def __init__(self, base_url: str, template: str = "default", api_key: str | None = None, request_timeout_s: float = 30.0) -> None:
        self.base_url = base_url.rstrip("/")
        self.template = template
        self.headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}
        self.request_timeout_s = request_timeout_s
        self.sandbox_id: str | None = None
        self.process = None

    def _post(self, path: str, body: dict, timeout: float) -> dict:
        import requests

        r = requests.post(self.base_url + path, json=body, headers=self.headers, timeout=timeout)
        r.raise_for_status()
        return r.json()

    async def start(self, command: str, cwd: Path) -> None:
        raise NotImplementedError("remote sandboxes run commands synchronously: use run()")

    async def ensure_sandbox(self, timeout_s: float = 600.0) -> str:
        if self.sandbox_id is None:
            out = await asyncio.to_thread(self._post, "/sandboxes", {"template": self.template, "timeout_s": timeout_s}, self.request_timeout_s)
            self.sandbox_id = out["id"]
        return self.sandbox_id

    async def run(self, command: str, cwd: Path, *, timeout_seconds: float | None = None) -> tuple[int, str]:
        sid = await self.ensure_sandbox()
        t = timeout_seconds or 600.0
        out = await asyncio.to_thread(self._post, f"/sandboxes/{sid}/exec", {"command": command, "cwd": str(cwd), "timeout_s": t},
                                      t + self.request_timeout_s)
        if out.get("timed_out"):
            raise TimeoutError(f"remote command timed out after {t}s")
        return int(out["exit_code"]), str(out.get("output", ""))

    async def terminate(self, *, timeout_seconds: float = DEFAULT_TERMINATE_TIMEOUT_SECONDS) -> None:
        if self.sandbox_id is None:
            return
        import requests

        sid, self.sandbox_id = self.sandbox_id, None
        try:
            await asyncio.to_thread(requests.delete, f"{self.base_url}/sandboxes/{sid}", headers=self.headers, timeout=timeout_seconds)
        except requests.RequestException:
            pass

"""Public tunnel to a local port (reference ``axrl/utils/tunnel.py:37-196``): black-box agents that
run outside this machine (remote sandboxes) reach the OpenAI proxy through a tunnel process such as
``cloudflared tunnel --url http://127.0.0.1:{port}``.  The command is a template; the tunnel is
ready once a line of its output matches ``ready_url_regex`` (the public base URL).  Its output
keeps being drained in the background so the process never blocks on a full pipe.
"""

from __future__ import annotations

import asyncio
import contextlib
import logging
import re
import shutil
import socket
from typing import Any, Mapping, Sequence

from pydantic import Field

from axrl_b200.configs import StrictBaseModel

logger = logging.getLogger(__name__)


class TunnelConfig(StrictBaseModel):
    command: list[str] = Field(default_factory=lambda: ["cloudflared", "tunnel", "--url", "http://127.0.0.1:{port}"])
    ready_url_regex: str = r"https://[-a-zA-Z0-9.]+\.trycloudflare\.com"
    startup_timeout_seconds: float = 30.0


def render_command(parts: Sequence[str], values: Mapping[str, Any]) -> list[str]:
    return [p.format(**values) for p in parts]


class Tunnel:
    def __init__(self, proc: asyncio.subprocess.Process, base_url: str, lines: list[str]) -> None:
        self.process, self.base_url, self.lines = proc, base_url.rstrip("/"), lines
        self._drain: asyncio.Task | None = None

    @classmethod
    async def start(cls, config: TunnelConfig, *, template_vars: Mapping[str, Any]) -> "Tunnel":
        cmd = render_command(config.command, template_vars)
        if not cmd:
            raise ValueError("tunnel command must be non-empty")
        if shutil.which(cmd[0]) is None:
            raise FileNotFoundError(f"tunnel executable {cmd[0]!r} not found")
        proc = await asyncio.create_subprocess_exec(*cmd, stdout=asyncio.subprocess.PIPE, stderr=asyncio.subprocess.STDOUT)
        lines: list[str] = []
        pat = re.compile(config.ready_url_regex)

        async def first_url() -> str:
            assert proc.stdout is not None
            while True:
                raw = await proc.stdout.readline()
                if not raw:
                    raise RuntimeError("tunnel process exited before printing its URL:\n" + "\n".join(lines[-20:]))
                line = raw.decode("utf-8", errors="replace").rstrip("\n")
                lines.append(line)
                m = pat.search(line)
                if m:
                    return m.group(0)

        t = cls(proc, "", lines)
        try:
            t.base_url = (await asyncio.wait_for(first_url(), config.startup_timeout_seconds)).rstrip("/")
        except BaseException:
            await t.stop()
            raise
        t._drain = asyncio.create_task(t._drain_output())
        return t

    async def _drain_output(self) -> None:
        assert self.process.stdout is not None
        while True:
            raw = await self.process.stdout.readline()
            if not raw:
                return
            self.lines.append(raw.decode("utf-8", errors="replace").rstrip("\n"))

    async def stop(self) -> None:
        if self._drain is not None:
            self._drain.cancel()
            with contextlib.suppress(asyncio.CancelledError):
                await self._drain
        if self.process.returncode is not None:
            return
        self.process.terminate()
        try:
            await asyncio.wait_for(self.process.wait(), 5.0)
        except asyncio.TimeoutError:
            self.process.kill()
            await self.process.wait()


def local_ip() -> str:
    """The address other machines reach this one at (the interface of the default route)."""
    with contextlib.closing(socket.socket(socket.AF_INET, socket.SOCK_DGRAM)) as s:
        try:
            s.connect(("10.255.255.255", 1))  # no packet is sent: only selects the outgoing interface
            return str(s.getsockname()[0])
        except OSError:
            return "127.0.0.1"

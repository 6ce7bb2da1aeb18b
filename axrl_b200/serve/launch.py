"""Launch engine servers (one per GPU or engine group) plus a router as child processes, wait
until they answer ``/health``, and stop them as process groups.

Reference: ``axrl/utils/sglang_launch_utils.py:222-286`` (standalone servers + ``sglang_router``
for the OPD teacher).
"""

from __future__ import annotations

import os
import signal
import subprocess
import sys
import time
from dataclasses import dataclass, field

from axrl_b200.utils.network_utils import get_free_port


@dataclass
class ServerGroup:
    procs: list[subprocess.Popen] = field(default_factory=list)
    urls: list[str] = field(default_factory=list)
    router_url: str | None = None

    def stop(self, timeout_s: float = 10.0) -> None:
        for p in self.procs:
            try:
                os.killpg(p.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
        t0 = time.time()
        for p in self.procs:
            try:
                p.wait(timeout=max(0.1, timeout_s - (time.time() - t0)))
            except subprocess.TimeoutExpired:
                try:
                    os.killpg(p.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass


def _wait_healthy(url: str, proc: subprocess.Popen, timeout_s: float) -> None:
    import requests

    t0 = time.time()
    while time.time() - t0 < timeout_s:
        if proc.poll() is not None:
            raise RuntimeError(f"server for {url} exited with code {proc.returncode}")
        try:
            if requests.get(url + "/health", timeout=2).ok:
                return
        except requests.RequestException:
            pass
        time.sleep(0.3)
    raise TimeoutError(f"{url} did not become healthy within {timeout_s}s")


def launch_servers(preset: str, devices: list[str], *, router: bool = True, host: str = "127.0.0.1", extra_args: list[str] | None = None,
                   timeout_s: float = 600.0) -> ServerGroup:
    g = ServerGroup()
    try:
        for dev in devices:
            port = get_free_port(host)
            env = dict(os.environ)
            cmd = [sys.executable, "-m", "axrl_b200.serve.engine_server", "--preset", preset, "--host", host, "--port", str(port),
                   "--device", dev] + (extra_args or [])
            g.procs.append(subprocess.Popen(cmd, env=env, start_new_session=True))
            g.urls.append(f"http://{host}:{port}")
        for u, p in zip(g.urls, g.procs):
            _wait_healthy(u, p, timeout_s)
        if router:
            port = get_free_port(host)
            cmd = [sys.executable, "-m", "axrl_b200.serve.router", "--backends", ",".join(g.urls), "--host", host, "--port", str(port)]
            g.procs.append(subprocess.Popen(cmd, start_new_session=True))
            g.router_url = f"http://{host}:{port}"
            _wait_healthy(g.router_url, g.procs[-1], 60.0)
    except Exception:
        g.stop()
        raise
    return g

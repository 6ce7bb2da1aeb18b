"""Command runners: output/exit code, timeout, and that terminating kills the command's whole
process tree (cf. the reference's CgroupRunner / E2BRunner, ``axrl/runner/*.py``)."""

import asyncio
import json
import os
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

import pytest

from axrl_b200.runner import CgroupRunner, ProcessGroupRunner, RemoteSandboxRunner


def test_process_group_runner_output_and_timeout(tmp_path):
    rc, out = asyncio.run(ProcessGroupRunner().run("echo hello; exit 3", tmp_path))
    assert rc == 3 and out.strip() == "hello"

    r = ProcessGroupRunner()

    async def go():
        with pytest.raises(TimeoutError):
            await r.run("sleep 30 & sleep 30", tmp_path, timeout_seconds=0.3)

    asyncio.run(go())
    pgid = r.process.pid
    with pytest.raises(ProcessLookupError):
        os.killpg(pgid, 0)  # the background child died with the group


@pytest.mark.skipif(not CgroupRunner.is_supported(), reason="no writable cgroup v2 hierarchy here")
def test_cgroup_runner_kills_escaped_children(tmp_path):
    rc, out = asyncio.run(CgroupRunner(memory_limit_bytes=1 << 30).run("setsid sleep 30 & echo started", tmp_path, timeout_seconds=10))
    assert rc == 0 and "started" in out


class _FakeSandbox(BaseHTTPRequestHandler):
    boxes: dict = {}

    def _json(self, code, obj):  # noqa: ANN001
        body = json.dumps(obj).encode()
        self.send_response(code)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def do_POST(self):  # noqa: N802
        body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
        if self.path == "/sandboxes":
            sid = f"sb{len(self.boxes)}"
            self.boxes[sid] = []
            return self._json(200, {"id": sid})
        sid = self.path.split("/")[2]
        self.boxes[sid].append(body["command"])
        return self._json(200, {"exit_code": 0, "output": f"ran {body['command']}"})

    def do_DELETE(self):  # noqa: N802
        self.boxes.pop(self.path.split("/")[2], None)
        self._json(200, {})

    def log_message(self, *a):  # noqa: ANN002
        pass


def test_remote_sandbox_runner_protocol(tmp_path):
    srv = HTTPServer(("127.0.0.1", 0), _FakeSandbox)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        r = RemoteSandboxRunner(f"http://127.0.0.1:{srv.server_port}", api_key="k")

        async def go():
            a = await r.run("ls", tmp_path)
            b = await r.run("pwd", tmp_path)
            await r.terminate()
            return a, b

        a, b = asyncio.run(go())
        assert a == (0, "ran ls") and b == (0, "ran pwd") and not _FakeSandbox.boxes
    finally:
        srv.shutdown()

"""Runner that places the command in its own cgroup v2, so terminate() stops every process it
spawned — including ones that left the session — and memory can be capped.

Reference: ``CgroupRunner`` (``axrl/runner/cgroup_runner.py:21-247``).  Here the runner uses a
writable cgroup v2 hierarchy (``AXRL_CGROUP_ROOT`` or ``/sys/fs/cgroup``): it creates a child
cgroup, starts the command paused behind a go-file, moves the command's pid into the cgroup,
sets ``memory.max`` and lets it run.  Terminate writes ``cgroup.kill`` (or SIGKILLs every pid in
``cgroup.procs`` on kernels without it) and removes the cgroup.  :meth:`is_supported` reports
whether the hierarchy is writable; callers fall back to the process-group runner otherwise.
"""

from __future__ import annotations

import asyncio
import os
import signal
import subprocess
import tempfile
import time
import uuid
from pathlib import Path

from axrl_b200.runner.base_runner import DEFAULT_TERMINATE_TIMEOUT_SECONDS, BaseRunner


def _root() -> Path:
    return Path(os.environ.get("AXRL_CGROUP_ROOT", "/sys/fs/cgroup"))


class CgroupRunner(BaseRunner):
    def __init__(self, name: str | None = None, memory_limit_bytes: int | None = None) -> None:
        if memory_limit_bytes is not None and memory_limit_bytes <= 0:
            raise ValueError("memory_limit_bytes must be > 0")
        self.name = f"{name or 'axrl'}-{uuid.uuid4().hex[:8]}"
        self.memory_limit_bytes = memory_limit_bytes
        self.process = None
        self.path: Path | None = None
        self._tmp: Path | None = None

    @staticmethod
    def is_supported() -> bool:
        root = _root()
        if not (root / "cgroup.controllers").exists():
            return False
        probe = root / f"axrl-probe-{uuid.uuid4().hex[:6]}"
        try:
            probe.mkdir()
            probe.rmdir()
            return True
        except OSError:
            return False

    async def start(self, command: str, cwd: Path) -> None:
        assert self.process is None, "a runner starts one command"
        if not self.is_supported():
            raise RuntimeError("CgroupRunner needs a writable cgroup v2 hierarchy (set AXRL_CGROUP_ROOT)")
        self.path = _root() / self.name
        self.path.mkdir()
        if self.memory_limit_bytes is not None and (self.path / "memory.max").exists():
            (self.path / "memory.max").write_text(str(self.memory_limit_bytes))
        self._tmp = Path(tempfile.mkdtemp(prefix="axrl-cg-"))
        go = self._tmp / "go"
        # the wrapper waits until it has been moved into the cgroup, then execs the command
        wrapper = f'while [ ! -e "{go}" ]; do sleep 0.01; done; exec bash -c {_shq(command)}'
        self.process = subprocess.Popen(["bash", "-c", wrapper], cwd=str(cwd), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                        start_new_session=True)
        try:
            (self.path / "cgroup.procs").write_text(f"{self.process.pid}\n")
            go.touch()
        except Exception:
            await self.terminate()
            raise

    def _pids(self) -> list[int]:
        try:
            return [int(x) for x in (self.path / "cgroup.procs").read_text().split()]
        except (OSError, ValueError):
            return []

    async def terminate(self, *, timeout_seconds: float = DEFAULT_TERMINATE_TIMEOUT_SECONDS) -> None:
        if self.path is None:
            return
        kill = self.path / "cgroup.kill"
        if kill.exists():
            try:
                kill.write_text("1")
            except OSError:
                pass
        for pid in self._pids():
            try:
                os.kill(pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
        t0 = time.time()
        while self._pids() and time.time() - t0 < timeout_seconds:
            await asyncio.sleep(0.02)
        if self.process is not None:
            try:
                self.process.wait(timeout=timeout_seconds)
            except subprocess.TimeoutExpired:
                pass
        try:
            self.path.rmdir()
        except OSError:
            pass
        self.path = None


def _shq(s: str) -> str:
    return "'" + s.replace("'", "'\"'\"'") + "'"

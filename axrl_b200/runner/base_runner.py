"""Runner interface and the process-group runner.

Reference: ``BaseRunner`` / ``CgroupRunner`` / ``E2BRunner`` (``axrl/runner/*.py``).  A runner
starts a shell command for an environment step, streams or collects its output, and guarantees
that terminating it also stops everything the command spawned.  :class:`ProcessGroupRunner` puts
the command in a new session and signals the whole process group (SIGTERM, then SIGKILL after a
grace period); :class:`~axrl_b200.runner.cgroup_runner.CgroupRunner` additionally catches
processes that leave the session (daemons, tmux) and applies a memory limit.  Neither is a
security sandbox.
"""

from __future__ import annotations

import asyncio
import os
import signal
import subprocess
import time
from pathlib import Path

DEFAULT_TERMINATE_TIMEOUT_SECONDS = 5.0


class BaseRunner:
    process: subprocess.Popen | None = None

    async def start(self, command: str, cwd: Path) -> None:
        raise NotImplementedError

    async def terminate(self, *, timeout_seconds: float = DEFAULT_TERMINATE_TIMEOUT_SECONDS) -> None:
        raise NotImplementedError

    async def run(self, command: str, cwd: Path, *, timeout_seconds: float | None = None) -> tuple[int, str]:
        """Run to completion; return (exit code, merged stdout+stderr).  TimeoutError on timeout
        (the command and its children are terminated first)."""
        await self.start(command, cwd)
        try:
            assert self.process is not None
            try:
                out, _ = await asyncio.to_thread(self.process.communicate, timeout=timeout_seconds)
            except subprocess.TimeoutExpired as e:
                raise TimeoutError(f"command timed out after {timeout_seconds}s") from e
            return int(self.process.returncode), out.decode(errors="replace")
        finally:
            await self.terminate()

    @property
    def returncode(self) -> int | None:
        return None if self.process is None else self.process.poll()


class ProcessGroupRunner(BaseRunner):
    def __init__(self, memory_limit_bytes: int | None = None) -> None:
        self.memory_limit_bytes = memory_limit_bytes
        self.process = None

    def _preexec(self):  # noqa: ANN202
        limit = self.memory_limit_bytes
        if limit is None:
            return None

        def fn() -> None:
            import resource

            resource.setrlimit(resource.RLIMIT_AS, (limit, limit))

        return fn

    async def start(self, command: str, cwd: Path) -> None:
        assert self.process is None, "a runner starts one command"
        self.process = subprocess.Popen(["bash", "-c", command], cwd=str(cwd), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                        start_new_session=True, preexec_fn=self._preexec())

    async def terminate(self, *, timeout_seconds: float = DEFAULT_TERMINATE_TIMEOUT_SECONDS) -> None:
        p = self.process
        if p is None:
            return
        pgid = p.pid  # session leader: its pid is the process-group id
        for sig, wait in ((signal.SIGTERM, timeout_seconds), (signal.SIGKILL, timeout_seconds)):
            try:
                os.killpg(pgid, sig)
            except ProcessLookupError:
                break
            t0 = time.time()
            while time.time() - t0 < wait:
                if p.poll() is not None and not _group_alive(pgid):
                    return
                await asyncio.sleep(0.05)


def _group_alive(pgid: int) -> bool:
    try:
        os.killpg(pgid, 0)
        return True
    except (ProcessLookupError, PermissionError):
        return False

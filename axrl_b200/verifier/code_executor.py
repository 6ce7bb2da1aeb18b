"""Run model-written Python solutions against test cases in a resource-limited subprocess.

Reference behaviour: ``axrl/verifier/leetcode_executor.py:23-196`` (unsafe_execute with a time
limit, swallowed I/O and a reliability guard).  Here each test runs the candidate in a fresh
``python -I`` child process with CPU-time, address-space and file-size rlimits, no inherited
environment, stdin fed from the test, in its own session (killed as a group on timeout).  This is
process isolation for reward computation, not a security sandbox.
"""

from __future__ import annotations

import os
import resource
import signal
import subprocess
import sys
import tempfile
from dataclasses import dataclass


@dataclass
class TestResult:
    passed: bool
    status: str  # "passed" | "failed" | "timeout" | "error"
    stdout: str = ""
    stderr: str = ""


def _limits(cpu_s: float, mem_bytes: int):  # noqa: ANN202
    def fn() -> None:
        resource.setrlimit(resource.RLIMIT_CPU, (int(cpu_s) + 1, int(cpu_s) + 1))
        resource.setrlimit(resource.RLIMIT_AS, (mem_bytes, mem_bytes))
        resource.setrlimit(resource.RLIMIT_FSIZE, (1 << 20, 1 << 20))
        os.setsid()

    return fn


def run_python(code: str, stdin: str = "", timeout_s: float = 5.0, mem_bytes: int = 1 << 30) -> TestResult:
    with tempfile.TemporaryDirectory(prefix="axrl-exec-") as d:
        path = os.path.join(d, "main.py")
        with open(path, "w") as f:
            f.write(code)
        p = subprocess.Popen([sys.executable, "-I", path], cwd=d, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                             env={"PATH": "/usr/bin:/bin"}, preexec_fn=_limits(timeout_s, mem_bytes))
        try:
            out, err = p.communicate(stdin.encode(), timeout=timeout_s)
        except subprocess.TimeoutExpired:
            try:
                os.killpg(p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            p.communicate()
            return TestResult(False, "timeout")
        if p.returncode != 0:
            return TestResult(False, "error", out.decode(errors="replace"), err.decode(errors="replace")[-2000:])
        return TestResult(True, "passed", out.decode(errors="replace"))


def check_io_tests(code: str, tests: list[tuple[str, str]], timeout_s: float = 5.0) -> tuple[float, list[TestResult]]:
    """Fraction of (stdin, expected stdout) tests whose output matches (whitespace-trimmed)."""
    results = []
    for inp, expected in tests:
        r = run_python(code, inp, timeout_s)
        if r.status == "passed" and r.stdout.strip() != expected.strip():
            r = TestResult(False, "failed", r.stdout, r.stderr)
        results.append(r)
    return (sum(r.passed for r in results) / max(1, len(results))), results


def check_assert_tests(code: str, test_code: str, timeout_s: float = 5.0) -> TestResult:
    """Run the solution followed by assertion-style tests; passes when the program exits 0."""
    return run_python(code + "\n\n" + test_code + "\n", "", timeout_s)

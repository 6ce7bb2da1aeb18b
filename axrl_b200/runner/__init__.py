"""Command runners for agent environments (tool execution, sandboxes)."""

from axrl_b200.runner.base_runner import BaseRunner, ProcessGroupRunner  # noqa: F401
from axrl_b200.runner.cgroup_runner import CgroupRunner  # noqa: F401
from axrl_b200.runner.remote_runner import RemoteSandboxRunner  # noqa: F401

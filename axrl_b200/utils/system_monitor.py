"""Host resource metrics and a background monitor thread.

Reference: ``axrl/utils/system_utils.py:78-300`` (FD / memory / disk / Ray-status metrics thread)
and ``PipelineController.start_resource_monitor`` (``axrl/pipeline/controller.py:1251-1287``).
Metrics come straight from ``/proc`` and ``statvfs``; GPU memory from the CUDA caching allocator
and ``torch.cuda.mem_get_info`` (no NVML calls that change state).
"""

from __future__ import annotations

import os
import threading
import time
from typing import Callable

import torch


def process_metrics(pid: int | None = None) -> dict[str, float]:
    pid = pid or os.getpid()
    out: dict[str, float] = {}
    try:
        out["system/process_open_fds"] = float(len(os.listdir(f"/proc/{pid}/fd")))
    except OSError:
        pass
    try:
        with open(f"/proc/{pid}/status") as f:
            for line in f:
                if line.startswith(("VmRSS:", "VmHWM:", "Threads:")):
                    k, v = line.split(":", 1)
                    val = float(v.split()[0])
                    out[f"system/process_{k.lower()}"] = val * 1024 if k.startswith("Vm") else val
    except OSError:
        pass
    return out


def host_metrics(disk_paths: tuple[str, ...] = ("/", "/tmp")) -> dict[str, float]:
    out: dict[str, float] = {}
    try:
        mem = {}
        with open("/proc/meminfo") as f:
            for line in f:
                k, v = line.split(":", 1)
                mem[k] = float(v.split()[0]) * 1024
        out["system/mem_total_bytes"] = mem.get("MemTotal", 0.0)
        out["system/mem_available_bytes"] = mem.get("MemAvailable", 0.0)
        out["system/mem_used_frac"] = 1.0 - mem.get("MemAvailable", 0.0) / max(mem.get("MemTotal", 1.0), 1.0)
    except OSError:
        pass
    try:
        with open("/proc/loadavg") as f:
            out["system/load_1m"] = float(f.read().split()[0])
    except OSError:
        pass
    try:
        with open("/proc/sys/fs/file-nr") as f:
            out["system/open_files_total"] = float(f.read().split()[0])
    except OSError:
        pass
    for p in disk_paths:
        try:
            st = os.statvfs(p)
            tag = p.strip("/").replace("/", "_") or "root"
            out[f"system/disk_{tag}_free_bytes"] = float(st.f_bavail * st.f_frsize)
            out[f"system/disk_{tag}_used_frac"] = 1.0 - st.f_bavail / max(st.f_blocks, 1)
        except OSError:
            pass
    return out


def gpu_metrics() -> dict[str, float]:
    if not torch.cuda.is_available():
        return {}
    out = {}
    for d in range(torch.cuda.device_count()):
        try:
            free, total = torch.cuda.mem_get_info(d)
        except RuntimeError:
            continue
        out[f"gpu{d}/mem_used_bytes"] = float(total - free)
        out[f"gpu{d}/torch_allocated_bytes"] = float(torch.cuda.memory_allocated(d))
        out[f"gpu{d}/torch_max_allocated_bytes"] = float(torch.cuda.max_memory_allocated(d))
        out[f"gpu{d}/torch_reserved_bytes"] = float(torch.cuda.memory_reserved(d))
    return out


class ResourceMonitor:
    """Samples process/host/GPU metrics every ``interval_s`` on a daemon thread and hands each
    sample to ``sink`` (e.g. a metric logger)."""

    def __init__(self, sink: Callable[[dict[str, float]], None], interval_s: float = 30.0, gpu: bool = True) -> None:
        self.sink, self.interval_s, self.gpu = sink, interval_s, gpu
        self._stop = threading.Event()
        self._th: threading.Thread | None = None
        self.samples = 0

    def sample(self) -> dict[str, float]:
        m = {**process_metrics(), **host_metrics()}
        if self.gpu:
            m.update(gpu_metrics())
        m["system/timestamp"] = time.time()
        return m

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                self.sink(self.sample())
                self.samples += 1
            except Exception:  # noqa: BLE001 - monitoring must never kill the job
                pass
            self._stop.wait(self.interval_s)

    def start(self) -> "ResourceMonitor":
        self._th = threading.Thread(target=self._loop, name="axrl-resource-monitor", daemon=True)
        self._th.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._th is not None:
            self._th.join(timeout=5)

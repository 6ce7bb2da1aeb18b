"""Loader for the in-tree sm_100a extension ``axrl_b200/_C*.so``.

The extension is compiled ahead of time by ``axrl_b200/csrc/build.py`` (called
from ``__graft_entry__.build``).  On a machine with a GPU every op dispatches
CUDA tensors to it.  If the shared object is missing there, the loader builds it
in-tree once (under a file lock, so concurrent ranks build it one time; set
``AXRL_AUTOBUILD=0`` to disable) and raises if that fails: no op silently falls
back to PyTorch.  CPU tensors use the PyTorch reference code in each
op module (the numerical oracle and the path CPU tests exercise).
"""

from __future__ import annotations

import glob
import importlib.util
import os
from types import ModuleType

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_MOD: ModuleType | None = None
_ERR: str | None = None


def _so_path(name: str) -> str | None:
    hits = sorted(glob.glob(os.path.join(_PKG_DIR, f"{name}*.so")))
    return hits[0] if hits else None


def _build_locked(name: str) -> str | None:
    """Build the missing extension in-tree; one process builds while the others wait on the lock."""
    import fcntl
    import sys

    from axrl_b200.csrc import build as _b

    os.makedirs(_b.BUILD, exist_ok=True)
    with open(os.path.join(_b.BUILD, ".lock"), "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            if _so_path(name) is None:
                sys.stderr.write(f"axrl_b200: extension {name} missing, building it in-tree\n")
                _b.build(only=name)
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)
    return _so_path(name)


def load(name: str = "_C") -> ModuleType:
    global _MOD, _ERR
    if _MOD is not None and name == "_C":
        return _MOD
    import torch  # noqa: F401  (libtorch symbols must be loaded first)

    path = _so_path(name)
    if path is None and torch.cuda.is_available() and os.environ.get("AXRL_AUTOBUILD", "1") != "0":
        path = _build_locked(name)
    if path is None:
        _ERR = f"extension {name} not built: run `python -m axrl_b200.csrc.build`"
        raise RuntimeError(_ERR)
    spec = importlib.util.spec_from_file_location(f"axrl_b200.{name}", path)
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    if name == "_C":
        _MOD = mod
    return mod


# Kernel launches per extension entry point (entry points not listed launch one kernel).
_KERNELS_PER_CALL = {"attn_bwd": 3, "paged_decode_attn": 2, "rmsnorm_bwd": 2, "logprob_fwd": 1, "gemm": 1, "sample_tokens": 2}
_COUNT = {"launches": 0, "enabled": False}


class _Counting:
    """Proxy over the extension module that tallies kernel launches while enabled."""

    def __init__(self, mod: ModuleType) -> None:
        self._mod = mod

    def __getattr__(self, name: str):  # noqa: ANN204
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*a, **k):  # noqa: ANN002, ANN003, ANN202
            if _COUNT["enabled"]:
                _COUNT["launches"] += _KERNELS_PER_CALL.get(name, 1)
            return fn(*a, **k)

        return wrapped

    @property
    def __file__(self) -> str:  # noqa: D401
        return self._mod.__file__


_PROXY: _Counting | None = None


def ext():  # noqa: ANN201
    """The CUDA extension (launch-counting proxy); raises loudly when absent."""
    global _PROXY
    if _PROXY is None:
        _PROXY = _Counting(load("_C"))
    return _PROXY


def count_launches(enabled: bool = True, reset: bool = False) -> int:
    if reset:
        _COUNT["launches"] = 0
    _COUNT["enabled"] = enabled
    return _COUNT["launches"]


def add_launches(n: int) -> None:
    """Graph replays re-launch the kernels captured once; callers add them here."""
    if _COUNT["enabled"]:
        _COUNT["launches"] += n


def available() -> bool:
    try:
        load("_C")
        return True
    except Exception:  # noqa: BLE001
        return False


def check_kernel_waits() -> None:
    """Raise if a kernel with bounded internal waits (tcgen05 attention forward / backward, the
    hand-written tcgen05 GEMM) gave up on a wait since the process started: its outputs are then
    incomplete.  Synchronises the stream."""
    e = ext()
    codes = {"tcgen05 attention": int(e.attn_tc_error()), "tcgen05 attention backward": int(e.attn_bwd_tc_error()),
             "tcgen05 GEMM": int(e.tc_linear_error())}
    bad = {k: v for k, v in codes.items() if v}
    if bad:
        raise RuntimeError(f"kernel wait timed out: {bad}")

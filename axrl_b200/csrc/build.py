"""Ahead-of-time build of the native extensions, in-tree.

* ``axrl_b200/_C*.so``       – CUDA kernels for sm_100a (+ torch bindings)
* ``axrl_b200/_runtime*.so`` – host C++ runtime: paged-KV block manager and radix
  prefix index, shared-memory tensor store, VMM tagged allocator

Objects are compiled in parallel with nvcc/g++ directly (no JIT cache outside
the tree), each only when its source or a header changed.  Every CUDA
translation unit is compiled with ``-gencode arch=compute_100a,code=sm_100a``.

Build time is dominated by header parsing, so kernel units include no torch
headers (``cuda_common.cuh``) or only the light ATen ones (``common.cuh``);
only ``bindings.cpp`` pulls in the Python module machinery.  Units are started
most expensive first (the CUTLASS GEMM instantiations, then the bindings) so the
cheap ones fill the remaining cores instead of queueing behind them.  Per-unit
compile seconds are written to ``_build/timings.json``.

Usage: ``python -m axrl_b200.csrc.build [-j N] [--force]``
"""

from __future__ import annotations

import argparse
import glob
import hashlib
import json
import os
import re
import subprocess
import sys
import sysconfig
import time
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
BUILD = os.path.join(PKG, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cutlass_include() -> str:
    import importlib.util

    spec = importlib.util.find_spec("flashinfer")
    cands = []
    if spec is not None and spec.submodule_search_locations:
        cands.append(os.path.join(list(spec.submodule_search_locations)[0], "data", "cutlass", "include"))
    site = sysconfig.get_paths()["purelib"]
    cands += [os.path.join(site, "flashinfer", "data", "cutlass", "include"), os.path.join(site, "tilelang", "3rdparty", "cutlass", "include")]
    for c in cands:
        if os.path.isfile(os.path.join(c, "cutlass", "cutlass.h")):
            return c
    raise RuntimeError("CUTLASS headers not found")


def _pybind11_include() -> str:
    import pybind11

    return pybind11.get_include()


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension as ce

    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}"]
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    defs = [abi, "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C", "-DPYBIND11_COMPILER_TYPE=\"_gcc\"",
            "-DPYBIND11_STDLIB=\"_libstdcpp\"", "-DPYBIND11_BUILD_ABI=\"_cxxabi1018\""]
    link = [f"-L{libdir}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda", f"-Wl,-rpath,{libdir}"]
    return inc + defs, link


_INCLUDE = re.compile(rb'^\s*#\s*include\s*"([^"]+)"', re.M)


def _local_deps(path: str, seen: set[str]) -> None:
    """Transitive closure of quoted includes that resolve inside this source tree."""
    with open(path, "rb") as f:
        text = f.read()
    for inc in _INCLUDE.findall(text):
        name = inc.decode()
        for base in (os.path.dirname(path), HERE):
            cand = os.path.normpath(os.path.join(base, name))
            if os.path.isfile(cand) and cand.startswith(HERE):
                if cand not in seen:
                    seen.add(cand)
                    _local_deps(cand, seen)
                break


def _digest(path: str, extra: list[str]) -> str:
    h = hashlib.sha1()
    deps: set[str] = set()
    _local_deps(path, deps)
    for p in [path, *sorted(deps)]:
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(extra).encode())
    return h.hexdigest()[:16]


def _compile(src: str, flags: list[str], force: bool) -> str:
    base = os.path.relpath(src, HERE).replace(os.sep, "_")
    obj = object_path(src, flags)
    if os.path.exists(obj) and not force:
        return obj
    for stale in glob.glob(os.path.join(BUILD, f"{base}.*.o")):
        os.remove(stale)
    if src.endswith(".cu"):
        cmd = ["nvcc", *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "--expt-extended-lambda",
               "-Xcompiler", "-fPIC", "-Xptxas", "-v", "-DNDEBUG", *flags, "-c", src, "-o", obj + ".tmp"]
    else:
        cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-DNDEBUG", *flags, "-c", src, "-o", obj + ".tmp"]
    t0 = time.time()
    res = subprocess.run(cmd, capture_output=True, text=True)
    _TIMES[os.path.relpath(src, HERE)] = round(time.time() - t0, 1)
    log = os.path.join(BUILD, f"{base}.log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stderr[-6000:])
        raise RuntimeError(f"compile failed: {src} (log {log})")
    os.replace(obj + ".tmp", obj)
    return obj


_TIMES: dict[str, float] = {}


def _cost(src: str) -> float:
    """Rough compile cost used to start expensive units first."""
    with open(src, "rb") as f:
        text = f.read()
    deps: set[str] = set()
    _local_deps(src, deps)
    heavy = any(d.endswith("gemm_sm100.cuh") for d in deps) or b"cutlass/" in text
    if heavy:
        return 1000.0 + len(text) / 1000.0
    if b"torch/extension.h" in text:
        return 500.0
    torch_lite = any(d.endswith(os.sep + "common.cuh") and not d.endswith("cuda_common.cuh") for d in deps)
    return (100.0 if torch_lite else 0.0) + len(text) / 1000.0


def sources() -> dict[str, list[str]]:
    """Translation units of each extension."""
    k = os.path.join(HERE, "kernels")
    r = os.path.join(HERE, "runtime")
    return {"_C": sorted(glob.glob(os.path.join(k, "*.cu"))) + sorted(glob.glob(os.path.join(k, "*.cpp"))),
            "_runtime": sorted(glob.glob(os.path.join(r, "*.cpp"))) + sorted(glob.glob(os.path.join(r, "*.cu")))}


def _link(objs: list[str], out: str, link: list[str]) -> None:
    cmd = ["g++", "-shared", "-o", out + ".tmp", *objs, *link]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stderr[-4000:])
        raise RuntimeError(f"link failed: {out}")
    os.replace(out + ".tmp", out)


def targets() -> dict[str, tuple[list[str], list[str], list[str]]]:
    """Extension name -> (sources, compile flags, link flags)."""
    tflags, tlink = _torch_flags()
    cut = _cutlass_include()
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    srcs_of = sources()
    return {
        "_C": (srcs_of["_C"],
               [*tflags, f"-I{cut}", f"-I{os.path.join(os.path.dirname(cut), 'tools', 'util', 'include')}", f"-I{HERE}",
                f"-I{cuda_home}/include", "-DCUTLASS_ENABLE_GDC_FOR_SM100"],
               [*tlink, f"-L{cuda_home}/lib64", f"-L{cuda_home}/lib64/stubs", "-lcudart", "-lcuda", f"-Wl,-rpath,{cuda_home}/lib64"]),
        "_runtime": (srcs_of["_runtime"],
                     [f"-I{sysconfig.get_paths()['include']}", f"-I{_pybind11_include()}", f"-I{HERE}", f"-I{cuda_home}/include"],
                     [f"-L{cuda_home}/lib64", "-lcudart", "-lrt", f"-Wl,-rpath,{cuda_home}/lib64"]),
    }


def object_path(src: str, flags: list[str]) -> str:
    """Object file of ``src`` for the current sources and flags (content-addressed)."""
    base = os.path.relpath(src, HERE).replace(os.sep, "_")
    return os.path.join(BUILD, f"{base}.{_digest(src, flags)}.o")


def output_path(name: str) -> str:
    return os.path.join(PKG, name + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build(jobs: int | None = None, force: bool = False, only: str | None = None) -> list[str]:
    """Compile every unit of the selected extensions in one pool (most expensive first), then link."""
    os.makedirs(BUILD, exist_ok=True)
    jobs = jobs or max(1, os.cpu_count() or 1)
    tg = {n: t for n, t in targets().items() if (not only or n == only) and t[0]}
    units = [(s, n) for n, (srcs, _, _) in tg.items() for s in srcs]
    units.sort(key=lambda u: _cost(u[0]), reverse=True)
    with ThreadPoolExecutor(jobs) as ex:
        futs = {u: ex.submit(_compile, u[0], tg[u[1]][1], force) for u in units}
        done = {u: f.result() for u, f in futs.items()}
    built = []
    for name, (srcs, _, link) in tg.items():
        objs = [done[(s, name)] for s in srcs]
        out = output_path(name)
        stamp = out + ".inputs"
        key = "\n".join(sorted(objs))
        if force or not os.path.exists(out) or not os.path.exists(stamp) or open(stamp).read() != key:
            _link(objs, out, link)
            with open(stamp, "w") as f:
                f.write(key)
        if not os.path.isfile(out):
            raise RuntimeError(f"extension {name} was not produced at {out}")
        built.append(out)
    if _TIMES:
        with open(os.path.join(BUILD, "timings.json"), "w") as f:
            json.dump(dict(sorted(_TIMES.items(), key=lambda kv: -kv[1])), f, indent=1)
    return built


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    for p in build(a.j, a.force, a.only):
        print(p)

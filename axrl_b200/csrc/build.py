"""Ahead-of-time build of the native extensions, in-tree.

* ``axrl_b200/_C*.so``       – CUDA kernels for sm_100a (+ torch bindings)
* ``axrl_b200/_runtime*.so`` – host C++ runtime: paged-KV block manager and radix
  prefix index, shared-memory tensor store, VMM tagged allocator

Objects are compiled in parallel with nvcc/g++ directly (no JIT cache outside
the tree), each only when its source or a header changed.  Every CUDA
translation unit is compiled with ``-gencode arch=compute_100a,code=sm_100a``.

Usage: ``python -m axrl_b200.csrc.build [-j N] [--force]``
"""

from __future__ import annotations

import argparse
import glob
import hashlib
import os
import re
import subprocess
import sys
import sysconfig
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
    dig = _digest(src, flags)
    obj = os.path.join(BUILD, f"{base}.{dig}.o")
    if os.path.exists(obj) and not force:
        return obj
    for stale in glob.glob(os.path.join(BUILD, f"{base}.*.o")):
        os.remove(stale)
    if src.endswith(".cu"):
        cmd = ["nvcc", *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "--expt-extended-lambda",
               "-Xcompiler", "-fPIC", "-Xptxas", "-v", "-DNDEBUG", *flags, "-c", src, "-o", obj + ".tmp"]
    else:
        cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-DNDEBUG", *flags, "-c", src, "-o", obj + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(BUILD, f"{base}.log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stderr[-6000:])
        raise RuntimeError(f"compile failed: {src} (log {log})")
    os.replace(obj + ".tmp", obj)
    return obj


def _link(objs: list[str], out: str, link: list[str]) -> None:
    cmd = ["g++", "-shared", "-o", out + ".tmp", *objs, *link]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stderr[-4000:])
        raise RuntimeError(f"link failed: {out}")
    os.replace(out + ".tmp", out)


def build(jobs: int | None = None, force: bool = False, only: str | None = None) -> list[str]:
    os.makedirs(BUILD, exist_ok=True)
    tflags, tlink = _torch_flags()
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    cut = _cutlass_include()
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    built = []
    jobs = jobs or max(1, os.cpu_count() or 1)

    targets = {
        "_C": (sorted(glob.glob(os.path.join(HERE, "kernels", "*.cu"))) + sorted(glob.glob(os.path.join(HERE, "kernels", "*.cpp"))),
               [*tflags, f"-I{cut}", f"-I{os.path.join(os.path.dirname(cut), 'tools', 'util', 'include')}", f"-I{HERE}",
                f"-I{cuda_home}/include", "-DCUTLASS_ENABLE_GDC_FOR_SM100"],
               [*tlink, f"-L{cuda_home}/lib64", f"-L{cuda_home}/lib64/stubs", "-lcudart", "-lcuda", f"-Wl,-rpath,{cuda_home}/lib64"]),
        "_runtime": (sorted(glob.glob(os.path.join(HERE, "runtime", "*.cpp"))) + sorted(glob.glob(os.path.join(HERE, "runtime", "*.cu"))),
                     [f"-I{sysconfig.get_paths()['include']}", f"-I{_pybind11_include()}", f"-I{HERE}", f"-I{cuda_home}/include"],
                     [f"-L{cuda_home}/lib64", "-lcudart", "-lrt", f"-Wl,-rpath,{cuda_home}/lib64"]),
    }
    for name, (srcs, flags, link) in targets.items():
        if only and name != only:
            continue
        if not srcs:
            continue
        with ThreadPoolExecutor(jobs) as ex:
            objs = list(ex.map(lambda s: _compile(s, flags, force), srcs))
        out = os.path.join(PKG, name + suffix)
        stamp = out + ".inputs"
        key = "\n".join(sorted(objs))
        if force or not os.path.exists(out) or not os.path.exists(stamp) or open(stamp).read() != key:
            _link(objs, out, link)
            with open(stamp, "w") as f:
                f.write(key)
        built.append(out)
    return built


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    for p in build(a.j, a.force, a.only):
        print(p)

"""Build-system checks that run without a GPU.

The CUDA extension must build inside a bounded CPU window, so these tests pin the
properties that keep it fast and complete: every kernel / runtime source is a unit of
an extension, only the bindings unit includes the full torch extension header, and
when the extensions are present they are linked from the current sources.
"""

import glob
import os

import pytest

from axrl_b200.csrc import build as B


def test_every_source_is_a_unit():
    srcs = B.sources()
    for sub, name in (("kernels", "_C"), ("runtime", "_runtime")):
        on_disk = {p for ext in ("*.cu", "*.cpp") for p in glob.glob(os.path.join(B.HERE, sub, ext))}
        assert on_disk == set(srcs[name]), (sub, on_disk ^ set(srcs[name]))


def test_only_bindings_include_full_torch_header():
    heavy = []
    for p in glob.glob(os.path.join(B.HERE, "**", "*.*"), recursive=True):
        if p.endswith((".cu", ".cuh", ".h", ".cpp")):
            with open(p, encoding="utf-8") as f:
                if "torch/extension.h" in f.read():
                    heavy.append(os.path.relpath(p, B.HERE))
    assert heavy == [os.path.join("kernels", "bindings.cpp")], heavy


def test_cutlass_units_are_torch_free():
    """CUTLASS instantiations are the slowest units; they must not parse ATen as well."""
    for p in glob.glob(os.path.join(B.HERE, "kernels", "*.cu")):
        deps: set[str] = set()
        B._local_deps(p, deps)
        if any(d.endswith("gemm_sm100.cuh") for d in deps):
            assert not any(d.endswith(os.sep + "common.cuh") and not d.endswith("cuda_common.cuh") for d in deps), p


def test_expensive_units_start_first():
    srcs = B.sources()["_C"]
    order = sorted(srcs, key=B._cost, reverse=True)
    first = [os.path.basename(p) for p in order[:4]]
    assert "grouped_gemm.cu" in first or any(n.startswith("gemm_") for n in first), first


def test_built_extensions_match_sources():
    tg = B.targets()
    for name, (srcs, flags, _) in tg.items():
        out = B.output_path(name)
        if not os.path.isfile(out):
            pytest.skip(f"{name} not built in this checkout")
        with open(out + ".inputs") as f:
            linked = set(f.read().split("\n"))
        expected = {B.object_path(s, flags) for s in srcs}
        assert linked == expected, f"{name} is stale: rebuild with python -m axrl_b200.csrc.build"

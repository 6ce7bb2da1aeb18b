"""GEMM microbenchmark over decode/prefill/training shapes of the Qwen3-8B model.

python -m axrl_b200.benchmarks.gemm_bench [--variants auto,skinny,swapab,cutlass]
Times each variant with CUDA events after warm-up, flushing L2 between iterations by READING a
512 MB buffer (a write flush would leave ~126 MB of dirty lines whose write-back the timed kernel
would pay for), and reports TB/s of operand traffic and TFLOP/s.
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", default="auto,tma,skinny,swapab,cutlass,tcgemm,tcstream,tccluster")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--sweep-decomp", action="store_true", help="skinny shapes under every stream-K decomposition")
    ap.add_argument("--bwd", action="store_true", help="data- and weight-gradient GEMMs: CUTLASS vs the hand-written kernel")
    ap.add_argument("--ms", default="1,8,32,64,128,256,4096", help="comma-separated M values")
    ap.add_argument("--shapes", default="qkv,o,gate_up,down,lm_head")
    ap.add_argument("--chain", type=int, default=0,
                    help="time N back-to-back GEMMs on distinct weights (up to 6 GB), stream-ordered with programmatic "
                         "dependent launch as in a decode step, instead of single isolated launches")
    a = ap.parse_args()
    if a.chain:
        return bench_chain(a)
    if a.sweep_decomp:
        return sweep_decomp(a.iters)
    if a.bwd:
        return bench_bwd(a)
    from axrl_b200.ops import _ext

    e = _ext.ext()
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288), "lm_head": (151936, 4096)}
    shapes = {k: v for k, v in shapes.items() if k in a.shapes.split(",")}
    for M in [int(m) for m in a.ms.split(",")]:
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device="cuda").bfloat16()
            w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
            res = {"M": M, "shape": name, "N": N, "K": K}
            for v in a.variants.split(","):
                if v == "skinny" and M > 64:
                    continue
                if (v in ("swapab", "tcstream") and M > 64) or (v == "tccluster" and M > 128) or (v == "tma" and M > 32):
                    continue
                try:
                    if v == "auto":
                        fn = lambda: e.linear_fwd(x, w)  # noqa: E731
                    elif v == "tcgemm":  # hand-written persistent tcgen05 kernel (tcgemm.cu)
                        fn = lambda: e.tc_linear(x, w)  # noqa: E731
                    else:
                        fn = lambda v=v: e.linear_variant(x, w, v)  # noqa: E731
                    for _ in range(3):
                        fn()
                    ts = []
                    for _ in range(a.iters):
                        flush.sum()
                        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        s.record()
                        fn()
                        t.record()
                        t.synchronize()
                        ts.append(s.elapsed_time(t))
                    ms = sorted(ts)[len(ts) // 2]
                    bytes_ = 2 * (M * K + N * K + M * N)
                    res[v] = {"us": round(ms * 1000, 1), "TBps": round(bytes_ / ms / 1e9, 2), "TFLOPs": round(2 * M * N * K / ms / 1e9, 1)}
                except Exception as ex:  # noqa: BLE001
                    res[v] = str(ex)[:80]
            print(json.dumps(res), flush=True)


def bench_chain(a) -> None:  # noqa: ANN001
    """Per-GEMM time inside a stream-ordered chain: every GEMM reads the same activation rows and its
    own weight matrix (never the same weights twice in a row, so every weight byte comes from HBM);
    launches overlap through programmatic dependent launch as in the decode step."""
    from axrl_b200.ops import _ext

    e = _ext.ext()
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288), "lm_head": (151936, 4096)}
    shapes = {k: v for k, v in shapes.items() if k in a.shapes.split(",")}
    e.set_pdl(True)
    e.set_weights_static(True)
    try:
        for M in [int(m) for m in a.ms.split(",")]:
            for name, (N, K) in shapes.items():
                n = max(2, min(a.chain, (6 << 30) // (2 * N * K)))
                ws = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(n)]
                x = torch.randn(M, K, device="cuda").bfloat16()
                res = {"M": M, "shape": name, "N": N, "K": K, "chain": n}
                for v in a.variants.split(","):
                    if (v in ("skinny", "swapab", "tcstream") and M > 64) or (v == "tccluster" and M > 128) or (v == "tma" and M > 32):
                        continue
                    try:
                        if v == "auto":
                            fn = lambda w: e.linear_fwd(x, w)  # noqa: E731
                        else:
                            fn = lambda w, v=v: e.linear_variant(x, w, v)  # noqa: E731
                        for w in ws[:2]:
                            fn(w)
                        torch.cuda.synchronize()
                        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        s0.record()
                        for w in ws:
                            fn(w)
                        s1.record()
                        s1.synchronize()
                        ms = s0.elapsed_time(s1) / n
                        bytes_ = 2 * (M * K + N * K + M * N)
                        res[v] = {"us": round(ms * 1000, 1), "TBps": round(bytes_ / ms / 1e9, 2)}
                    except Exception as ex:  # noqa: BLE001
                        res[v] = str(ex)[:80]
                print(json.dumps(res), flush=True)
                del ws
                torch.cuda.empty_cache()
    finally:
        e.set_weights_static(False)


def bench_bwd(a) -> None:  # noqa: ANN001
    """dX = dY @ W and dW += dY^T @ X for the Qwen3-8B projections at M tokens."""
    from axrl_b200.ops import _ext

    e = _ext.ext()
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}
    for M in [int(m) for m in a.ms.split(",")]:
        for name, (N, K) in shapes.items():
            if name not in a.shapes.split(","):
                continue
            dy = torch.randn(M, N, device="cuda").bfloat16()
            w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
            x = torch.randn(M, K, device="cuda").bfloat16()
            acc = torch.zeros(N, K, device="cuda")
            fl = 2.0 * M * N * K
            res = {"M": M, "shape": name, "N": N, "K": K}
            for label, fn in (("dgrad_cutlass", lambda: e.linear_dgrad(dy, w)), ("dgrad_tc", lambda: e.tc_linear_dgrad(dy, w)),
                              ("wgrad_cutlass", lambda: e.linear_wgrad_acc(dy, x, acc)),
                              ("wgrad_tc", lambda: e.tc_linear_wgrad_acc(dy, x, acc, True))):
                ms = _time(fn, flush, a.iters)
                res[label] = {"us": round(ms * 1000, 1), "TFLOPs": round(fl / ms / 1e9, 1)}
            print(json.dumps(res), flush=True)


def _time(fn, flush: torch.Tensor, iters: int) -> float:
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        flush.sum()
        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        t.record()
        t.synchronize()
        ts.append(s.elapsed_time(t))
    return sorted(ts)[len(ts) // 2]


def sweep_decomp(iters: int) -> None:
    """Decode-sized GEMMs (swap-AB path) under heuristic / data-parallel / split-K / stream-K."""
    from axrl_b200.ops import _ext

    e = _ext.ext()
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}
    modes = [("heuristic", 0, 0), ("dp", 1, 0), ("split2", 2, 2), ("split4", 2, 4), ("split8", 2, 8), ("streamk", 3, 0)]
    for M in (8, 32, 64):
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device="cuda").bfloat16()
            w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
            ref = e.linear_variant(x, w, "skinny").float()
            res = {"M": M, "shape": name}
            for tag, mode, splits in modes:
                e.set_streamk_decomposition(mode, splits)
                try:
                    y = e.linear_variant(x, w, "swapab")
                    err = (y.float() - ref).abs().max().item()
                    ms = _time(lambda: e.linear_variant(x, w, "swapab"), flush, iters)
                    res[tag] = {"us": round(ms * 1000, 1), "TBps": round(2 * N * K / ms / 1e9, 2), "err": round(err, 4)}
                except Exception as ex:  # noqa: BLE001
                    res[tag] = str(ex)[:60]
            e.set_streamk_decomposition(0, 0)
            print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

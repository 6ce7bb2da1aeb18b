"""Packed causal attention (training / log-prob passes): forward and backward throughput.

Sequences of ``--lens`` tokens are packed into one buffer (Qwen3-8B heads: 32 q / 8 kv, head dim
128, bf16) and attended causally per sequence through the range-list kernels
(``csrc/kernels/attention.cu``).  Reference counterpart: the packed-attention cost inside ``benchmark/magi_forward`` (Magi
``calc_attn``, ``axrl/utils/megatron/magi_forward.py:439-466``).  Reports CUDA-event device time and TFLOP/s (causal FLOPs:
4 * D * Hq * sum(L * (L + 1) / 2) forward, 2.5x that backward).

python -m axrl_b200.benchmarks.attention_bench [--lens 8192,2048,2048,1024,1024,512,512] [--iters 5]
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--lens", default="8192,2048,2048,1024,1024,512,512,256,256")
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--no-bwd", action="store_true")
    a = ap.parse_args()
    from axrl_b200.ops import core
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    lens = [int(x) for x in a.lens.split(",")]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T, D = cu[-1], 128
    spec = causal_spec_from_cu_seqlens(cu).to("cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(T, a.hq, D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(T, a.hkv, D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    v = torch.randn(T, a.hkv, D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    do = torch.randn(T, a.hq, D, device="cuda", generator=g).bfloat16()
    flops_f = 4.0 * D * a.hq * sum(n * (n + 1) / 2 for n in lens)

    def timed(fn) -> float:  # noqa: ANN001
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / a.iters

    with torch.no_grad():
        f_ms = timed(lambda: core.attention(q, k, v, spec))
    out = {"tokens": T, "lens": lens, "hq": a.hq, "hkv": a.hkv, "fwd_ms": round(f_ms, 3), "fwd_tflops": round(flops_f / f_ms / 1e9, 1)}
    if not a.no_bwd:
        o = core.attention(q, k, v, spec)

        def bwd() -> None:
            torch.autograd.grad(o, (q, k, v), do, retain_graph=True)

        b_ms = timed(bwd)
        out.update({"bwd_ms": round(b_ms, 3), "bwd_tflops": round(2.5 * flops_f / b_ms / 1e9, 1)})
    print(json.dumps(out))


if __name__ == "__main__":
    main()

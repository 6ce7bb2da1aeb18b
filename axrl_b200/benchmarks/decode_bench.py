"""Rollout-engine microbenchmark: prefill + decode throughput of a Qwen3-shaped model.

python -m axrl_b200.benchmarks.decode_bench --model qwen3-8b --batch 256 --prompt 512 --new 256 [--pdl 0]
(AXRL_DECODE_GEMM=skinny|tma|tcgen05 forces the decode-size GEMM kernel.)  Reports device-timed prefill seconds, decode ms/step and decode tokens/s (CUDA events).
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--burst", type=int, default=16)
    ap.add_argument("--pdl", type=int, default=1, help="programmatic dependent launch of the decode kernels (0 = off)")
    a = ap.parse_args()
    import os

    from axrl_b200.ops import _ext

    _ext.ext().set_pdl(bool(a.pdl))

    from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    cfg = resolve_preset(a.model)
    with torch.device("cuda"):
        model = Qwen3Model(cfg).to(torch.bfloat16)
    model.init_weights(0)
    model.inv_freq = model.inv_freq.float()
    ctx = a.prompt + a.new + 64
    eng = RolloutEngine(model, max_batch=a.batch, kv_tokens=a.batch * (ctx + 64), max_context=ctx, use_cuda_graph=not a.eager,
                        burst=a.burst)

    def reqs(tag: str) -> list[GenRequest]:
        g = torch.Generator().manual_seed(0)
        out = []
        for p in range(a.batch // a.group):
            prompt = torch.randint(1, cfg.vocab_size, (a.prompt,), generator=g).tolist()
            out += [GenRequest(rid=f"{tag}{p}-{i}", prompt=prompt, max_new_tokens=a.new, forced_len=a.new, forced_token=0,
                               seed_stream=p * 100 + i) for i in range(a.group)]
        return out

    eng.generate(reqs("w"))  # warm-up: graph capture for every bucket on the way
    torch.cuda.synchronize()
    eng.stats = {k: 0 for k in eng.stats}
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    eng.generate(reqs("t"))
    e.record()
    torch.cuda.synchronize()
    total = s.elapsed_time(e) / 1000
    st = eng.stats
    print(json.dumps({"model": a.model, "batch": a.batch, "prompt": a.prompt, "new": a.new, "total_s": round(total, 3),
                      "prefill_s": round(st["prefill_s"], 3), "decode_s": round(st["decode_s"], 3),
                      "decode_ms_per_step": round(1000 * st["decode_s"] / max(1, st["decode_steps"]), 3),
                      "decode_tok_per_s": round(st["decode_tokens"] / max(1e-9, st["decode_s"]), 1), "bursts": st["bursts"],
                      "graph": not a.eager, "pdl": bool(a.pdl), "decode_gemm": os.environ.get("AXRL_DECODE_GEMM", "default")}))
    eng.release_graphs()


if __name__ == "__main__":
    main()

"""Weight-sync microbenchmark: trainer TP shards -> rollout engines, bf16 and block-fp8.

Reference: ``benchmark/weight_update/*.py`` (colocated timing, bf16-vs-fp8 sync).  Default layout
on 8 GPUs: a Qwen3-8B-shaped trainer with TP=4 on ranks 0-3 pushes to two rollout engines with
TP=2 on ranks 4-5 and 6-7.  Reports, per mode, seconds per full reshard + push (device-timed, max
over ranks), the bytes that cross NVLink and the achieved GB/s, for the fused P2P kernel and for
the NCCL-broadcast + local-reshard baseline.

torchrun --nproc-per-node 8 -m axrl_b200.benchmarks.weight_sync_bench [--model qwen3-8b] [--iters 5]
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--trainer-tp", type=int, default=None)
    ap.add_argument("--rollout-tp", type=int, default=None)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(minutes=5), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.sync.plan import qwen3_param_specs
    from axrl_b200.sync.weight_sync import WeightSyncer

    cfg = resolve_preset(a.model)
    specs = qwen3_param_specs(cfg)
    half = max(1, world // 2)
    ttp = a.trainer_tp or half
    rtp = a.rollout_tp or max(1, half // 2)
    src = list(range(ttp))
    dst_ranks = list(range(ttp, world)) if world > ttp else list(range(world))
    groups = [dst_ranks[i:i + rtp] for i in range(0, len(dst_ranks) - rtp + 1, rtp)]
    out = {"model": a.model, "world": world, "trainer_tp": ttp, "rollout_tp": rtp, "engines": len(groups)}
    for fp8 in (False, True):
        ws = WeightSyncer(specs, src_tp=ttp, src_ranks=src, dst_tp=rtp, dst_groups=groups, fp8=fp8)
        if ws.src_rank is not None:
            ws.src_view()[: ws.src_layout.nbytes // 2].normal_(0, 0.02)
        for name, fn in (("p2p", ws.push), ("nccl", ws.push_nccl)):
            for _ in range(a.warmup):
                fn()
            ts = [fn() for _ in range(a.iters)]
            t = torch.tensor([sorted(ts)[len(ts) // 2]], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            pushed = torch.tensor([float(ws.bytes_pushed)], device="cuda")
            dist.all_reduce(pushed)
            sec = float(t)
            key = f"{'fp8' if fp8 else 'bf16'}_{name}"
            out[key] = {"seconds": round(sec, 5), "bytes_to_destinations": int(pushed), "GBps": round(float(pushed) / sec / 1e9, 1)}
        del ws
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Fused compute + collective paths against their NCCL baselines, as a fraction of the roofline.

Run under torchrun, one rank per GPU (N = 2..8):

* ``tp``: tensor-parallel GEMMs of the Qwen3-8B MLP with sequence parallelism, T tokens:
  all-gather -> GEMM (``ag_linear``: (T/N, 4096) gathered, times the (2*12288/N, 4096) gate/up
  shard) and GEMM -> reduce-scatter (``linear_rs``: (T, 12288/N) times the (4096, 12288/N) down
  shard, rows reduce-scattered), NVLink P2P kernels (``parallel/tp_overlap.py``) vs NCCL
  all-gather / reduce-scatter around the same GEMM.
* ``ep``: one MoE layer of the Qwen3-30B-A3B shape (hidden 2048, 128 experts, top-8, expert FFN
  768) with EP=N: routing, dispatch, grouped expert FFN, combine; NVLink device-side
  dispatch/combine (``parallel/ep_p2p.py``) vs NCCL all-to-all (``parallel/expert.py``).

Reference counterparts: Megatron's TP + sequence-parallel linears and the ``alltoall`` MoE token
dispatcher (``axrl/worker/megatron_worker.py:833``), both on NCCL.

Roofline of a fused path: the slower of its FLOPs at the measured bf16 GEMM peak and the bytes
each GPU must receive over NVLink at the measured 770 GB/s per direction.  Every time is CUDA-event
device time, max over ranks, median of ``--iters`` after ``--warmup`` iterations.

torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m axrl_b200.benchmarks.fused_comm_bench [--paths tp,ep] [--tokens 16384]

``--paths kernels`` (one GPU, plain ``python -m``): the fused kernels alone, for profiler captures.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per GPU


def _peaks() -> tuple[float, float]:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk.get("bf16_tflops", 1590.0)), float(pk.get("hbm_gbs", 6650.0))
    except (OSError, ValueError):
        return 1590.0, 6650.0


def _time(fn, warmup: int, iters: int) -> float:  # noqa: ANN001
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(iters):
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ts.append(float(t))
    return statistics.median(ts)


def bench_tp(T: int, warmup: int, iters: int, tflops: float) -> list[dict]:
    from axrl_b200.parallel.tensor_parallel import TPContext, column_parallel_linear, row_parallel_linear

    N, r = dist.get_world_size(), dist.get_rank()
    H, F = 4096, 12288
    g = torch.Generator(device="cuda").manual_seed(11 + r)
    x_sp = torch.randn(T // N, H, device="cuda", generator=g).bfloat16()
    w_gu = (torch.randn(2 * F // N, H, device="cuda", generator=g) * 0.02).bfloat16()
    y = torch.randn(T, F // N, device="cuda", generator=g).bfloat16()
    w_dn = (torch.randn(H, F // N, device="cuda", generator=g) * 0.02).bfloat16()
    out = []
    ctxs = {b: TPContext.from_group(dist.group.WORLD, backend=b) for b in ("torch", "p2p")}
    # the GEMM -> reduce-scatter fused into one tcgen05 kernel storing tiles into the owners' slots
    os.environ["AXRL_TP_FUSED"] = "1"
    ctxs["p2p_fused"] = TPContext.from_group(dist.group.WORLD, backend="p2p")
    os.environ["AXRL_TP_FUSED"] = "0"
    ref_ag = column_parallel_linear(x_sp, w_gu, ctxs["torch"])
    ref_rs = row_parallel_linear(y, w_dn, ctxs["torch"])
    for name, fn, flops, nbytes, ref in (
        ("ag_gemm", column_parallel_linear, 2.0 * T * H * (2 * F // N), (N - 1) / N * T * H * 2, ref_ag),
        ("gemm_rs", row_parallel_linear, 2.0 * T * (F // N) * H, (N - 1) / N * T * H * 2, ref_rs),
    ):
        row = {"path": f"tp_{name}", "tokens": T, "n_gpus": N}
        for b, tp in ctxs.items():
            args = (x_sp, w_gu) if name == "ag_gemm" else (y, w_dn)
            res = fn(*args, tp)
            err = ((res.float() - ref.float()).abs().max() / (ref.float().abs().max() + 1e-6)).item()
            row[f"{b}_ms"] = round(_time(lambda: fn(*args, tp), warmup, iters), 4)  # noqa: B023
            row[f"{b}_rel_err"] = float(f"{err:.2e}")
        target_ms = max(flops / (tflops * 1e12), nbytes / (NVLINK_GBS * 1e9)) * 1e3
        row.update({"gflop": round(flops / 1e9, 1), "nvlink_mb_per_gpu": round(nbytes / 1e6, 1), "roofline_ms": round(target_ms, 4),
                    "p2p_frac_of_roofline": round(target_ms / row["p2p_ms"], 3),
                    "p2p_fused_frac_of_roofline": round(target_ms / row["p2p_fused_ms"], 3),
                    "nccl_frac_of_roofline": round(target_ms / row["torch_ms"], 3)})
        ctxs["p2p"].comm.check()
        ctxs["p2p_fused"].comm.check()
        out.append(row)
    return out


def bench_ep(T: int, warmup: int, iters: int, tflops: float) -> list[dict]:
    from axrl_b200.models.moe import MoEBlock
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.parallel.expert import EPContext

    N, r = dist.get_world_size(), dist.get_rank()
    cfg = resolve_preset("qwen3-30b-a3b")
    H, E, k, F = cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    g = torch.Generator(device="cuda").manual_seed(5 + r)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    out = []
    row = {"path": "ep_moe_layer", "tokens_per_gpu": T, "n_gpus": N, "experts": E, "top_k": k}
    results = {}
    for b in ("torch", "p2p"):
        ep = EPContext.from_group(dist.group.WORLD, backend=b, hidden=H, num_experts=E, max_rows=T * k)
        blk = MoEBlock(cfg, ep=ep).to("cuda", torch.bfloat16)
        torch.manual_seed(123)  # the same expert weights for both backends
        with torch.no_grad():
            for p in blk.parameters():
                p.normal_(0.0, 0.02)
        fn = lambda: blk(x)  # noqa: E731
        with torch.no_grad():
            results[b] = fn().float()
            row[f"{b}_ms"] = round(_time(fn, warmup, iters), 4)
        if hasattr(ep.comm, "check"):
            ep.comm.check()
        del blk
    ref = results["torch"]
    row["p2p_rel_err"] = float(f"{((results['p2p'] - ref).abs().max() / (ref.abs().max() + 1e-6)).item():.2e}")
    flops = 2.0 * T * k * 3 * H * F
    nbytes = 2 * (N - 1) / N * T * k * H * 2  # dispatch + combine rows that leave the GPU
    target_ms = max(flops / (tflops * 1e12), nbytes / (NVLINK_GBS * 1e9)) * 1e3
    row.update({"gflop": round(flops / 1e9, 1), "nvlink_mb_per_gpu": round(nbytes / 1e6, 1), "roofline_ms": round(target_ms, 4),
                "p2p_frac_of_roofline": round(target_ms / row["p2p_ms"], 3), "nccl_frac_of_roofline": round(target_ms / row["torch_ms"], 3)})
    out.append(row)
    return out


def bench_kernels_1gpu(T: int, warmup: int, iters: int, tflops: float, hbm_gbs: float) -> list[dict]:
    """The fused kernels on ONE GPU (world size 1), for a profiler capture of the kernel itself:
    the tcgen05 GEMM storing its tiles into the (here local) owner slots with the channel handshake,
    against the plain tcgen05 GEMM; the partitioned AdamW storing bf16 parameters through the
    pointer table, against the AdamW kernel with its local bf16 write-back."""
    from axrl_b200.ops import _ext
    from axrl_b200.parallel.tp_overlap import P2PTPComm

    e = _ext.ext()
    H, F = 4096, 12288
    g = torch.Generator(device="cuda").manual_seed(3)
    y = torch.randn(T, F // 2, device="cuda", generator=g).bfloat16()  # a TP=2 down-projection shard
    w = (torch.randn(H, F // 2, device="cuda", generator=g) * 0.02).bfloat16()
    os.environ["AXRL_TP_FUSED"] = "1"
    comm = P2PTPComm(dist.group.WORLD, cap_tokens=T, hidden=H)
    os.environ["AXRL_TP_FUSED"] = "0"
    ref = e.linear_fwd(y, w)
    got = comm.gemm_rs_fused(y, w, None)
    err = ((got.float() - ref.float()).abs().max() / (ref.float().abs().max() + 1e-6)).item()
    flops = 2.0 * T * (F // 2) * H
    rows = []
    t_plain = _time(lambda: e.linear_fwd(y, w), warmup, iters)
    t_fused = _time(lambda: comm.gemm_rs_fused(y, w, None), warmup, iters)
    comm.check()
    rows.append({"path": "gemm_to_slots_1gpu", "M": T, "N": H, "K": F // 2, "plain_ms": round(t_plain, 4), "fused_ms": round(t_fused, 4),
                 "plain_tflops": round(flops / t_plain / 1e9, 1), "fused_tflops": round(flops / t_fused / 1e9, 1), "rel_err": float(f"{err:.2e}")})
    n = 64 << 20  # 64 M parameters of one partition
    p = torch.randn(n, device="cuda", generator=g)
    gr = torch.randn(n, device="cuda", generator=g) * 1e-3
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    pb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    ptrs = torch.tensor([pb.data_ptr()], dtype=torch.int64, device="cuda")
    sq = (gr.pow(2).sum()).reshape(1)
    t_adam = _time(lambda: e.adamw_step(p, gr, m, v, pb, n, 1e-5, 0.9, 0.999, 1e-8, 0.01, 2, sq, 1.0, 1.0), warmup, iters)
    t_p2p = _time(lambda: e.adamw_p2p_step(p, gr, m, v, ptrs, 0, n, 1e-5, 0.9, 0.999, 1e-8, 0.01, 2, sq, 1.0, 1.0), warmup, iters)
    nbytes = n * (4 * 4 + 4 * 3 + 2)  # read p, g, m, v; write p, m, v and the bf16 parameter
    rows.append({"path": "adamw_param_store_1gpu", "params": n, "adamw_ms": round(t_adam, 4), "adamw_p2p_ms": round(t_p2p, 4),
                 "adamw_gbs": round(nbytes / t_adam / 1e6, 1), "adamw_p2p_gbs": round(nbytes / t_p2p / 1e6, 1),
                 "adamw_p2p_frac_of_hbm": round(nbytes / t_p2p / 1e6 / hbm_gbs, 3)})
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--paths", default="tp,ep")
    ap.add_argument("--tokens", type=int, default=16384, help="TP: tokens of the sequence-parallel batch")
    ap.add_argument("--ep-tokens", type=int, default=8192, help="EP: tokens per GPU")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    for k, val in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29561"), ("RANK", "0"), ("WORLD_SIZE", "1")):
        os.environ.setdefault(k, val)  # a plain ``python -m`` run is a one-rank job
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(minutes=5), device_id=torch.device("cuda", local))
    tflops, hbm = _peaks()
    rows = []
    paths = a.paths.split(",")
    if "tp" in paths:
        rows += bench_tp(a.tokens, a.warmup, a.iters, tflops)
    if "ep" in paths:
        rows += bench_ep(a.ep_tokens, a.warmup, a.iters, tflops)
    if "kernels" in paths:
        rows += bench_kernels_1gpu(a.tokens, a.warmup, a.iters, tflops, hbm)
    if dist.get_rank() == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

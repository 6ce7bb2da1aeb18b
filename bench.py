"""GRPO step benchmark: Qwen3-8B-shaped dense model, colocated rollout + trainer, bf16, random init.

Workload per GPU (weak scaling):
  prompts of 512 uniform-random token ids, group size 8; response lengths forced
  through EOS to a log-normal draw (median 1024, sigma 1.0, clipped to [16, 8192]);
  reward = 1 if token 7 appears; ref + old logprob recompute, one optimizer step
  (AdamW, fp32 master, ZeRO over the data-parallel ranks), colocated weight sync.
  Streaming partial rollout: `--inflight-per-gpu` groups stay in generation and a
  step trains the first `--prompts-per-gpu` groups to complete; unfinished groups
  keep their partial responses and resume after the weight update, so a step's
  rollout is bounded by throughput rather than by the longest response.
Metric: trained tokens per second for the whole job (prompt + response tokens of
every sequence trained in the step, summed over ranks) and seconds per GRPO step.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch with torch.distributed.run (one rank per GPU, NCCL).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GRPO step s & tokens/s/box (8B dense, 30B-A3B MoE) at 1/2/4/8 B200; sync s"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--prompts-per-gpu", type=int, default=4, help="groups trained per step per GPU")
    ap.add_argument("--inflight-per-gpu", type=int, default=16, help="groups kept in generation per GPU (partial rollout)")
    ap.add_argument("--no-partial", action="store_true", help="every step generates its own groups to completion")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--median", type=float, default=1024.0)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--mb-tokens", type=int, default=16384)
    ap.add_argument("--no-ref", action="store_true", help="skip the reference-policy logprob pass")
    ap.add_argument("--kv-gb", type=float, default=None, help="KV pool size (default: free memory minus --headroom-gb)")
    ap.add_argument("--headroom-gb", type=int, default=24)
    ap.add_argument("--tp", type=int, default=1, help="tensor parallelism (TP groups of consecutive ranks, data parallel across them)")
    ap.add_argument("--ep", type=int, default=None,
                    help="expert parallelism for MoE models (default: every GPU, dense parts data-parallel over the same ranks)")
    ap.add_argument("--ep-backend", choices=["p2p", "torch"], default="p2p", help="EP dispatch / combine: NVLink kernels or NCCL all-to-all")
    ap.add_argument("--deterministic", action="store_true", help="deterministic attention backward (separate dQ pass)")
    ap.add_argument("--verbose", action="store_true")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int) -> None:
        self.idx = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                                          "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def reference_arm(a) -> None:  # noqa: ANN001
    """The reference (XYZ-AI-Lab/axrl) needs SGLang + Megatron-Core + Ray, none of which exist offline here."""
    why = None
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "axrl")):
        why = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        missing = []
        for mod in ("sglang", "megatron.core", "ray", "transformer_engine", "tensordict"):
            try:
                __import__(mod)
            except Exception:  # noqa: BLE001
                missing.append(mod)
        if missing:
            why = f"reference GRPO path needs {', '.join(missing)}, not installable offline (no wheels, no network)"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why or "reference run path not wired"}), flush=True)


def main() -> None:
    a = _args()
    if a.impl == "reference":
        reference_arm(a)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(minutes=20), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.ops import _ext
    from axrl_b200.pipeline.grpo_step import SyntheticGRPO, SyntheticGRPOConfig
    from axrl_b200.train.engine import ParallelCtx, TrainEngine

    mcfg = resolve_preset(a.model)
    # deterministic_mode=False: the attention backward accumulates dQ with fp32 atomics (the
    # deterministic variant adds a separate dQ pass); stated in the printed config
    wc = MegatronWorkerConfig(recompute_granularity="full", max_tokens_per_micro_batch=a.mb_tokens, seed=1234,
                              deterministic_mode=a.deterministic)
    grpo = GrpoTrainerConfig(loss_type="grpo", mismatch_token_clip_max=2.0)
    ep = (a.ep or world) if mcfg.is_moe else 1
    if ep not in (1, world):
        raise SystemExit("--ep must be 1 or the number of GPUs")
    tp = a.tp
    if world % tp or (tp > 1 and mcfg.is_moe):
        raise SystemExit("--tp must divide the number of GPUs (dense models)")
    dp, dp_rank = world // tp, rank // tp
    if tp > 1:  # every rank creates every group, in the same order
        tp_groups = [dist.new_group(list(range(i, i + tp))) for i in range(0, world, tp)]
        dp_groups = [dist.new_group(list(range(j, world, tp))) for j in range(tp)]
        par = ParallelCtx(dp_group=dp_groups[rank % tp] if dp > 1 else None, dp_size=dp, dp_rank=dp_rank, tp_group=tp_groups[rank // tp],
                          tp_size=tp, tp_rank=rank % tp, tp_backend="p2p")
    else:
        par = ParallelCtx(dp_group=dist.group.WORLD if world > 1 else None, dp_size=world, dp_rank=rank,
                          ep_group=dist.group.WORLD if ep > 1 else None, ep_size=ep, ep_backend=a.ep_backend)
    train = TrainEngine(wc, mcfg, dev, par=par)
    train.optim.release_grads()  # gradients live only inside the train phase
    torch.cuda.empty_cache()  # the caching allocator still holds the released blocks
    free = torch.cuda.mem_get_info(dev)[0]
    # reference-policy weights on the device when that still leaves a 40 GB KV pool (a device copy
    # per step instead of a host-to-device copy of the whole model)
    ref_bytes = sum(p.numel() * p.element_size() for p in train.model.parameters())
    ref_dev = not a.no_ref and free - ref_bytes - (a.headroom_gb << 30) >= (40 << 30)
    kv_gb = a.kv_gb if a.kv_gb else max(2.0, (free - (ref_bytes if ref_dev else 0) - (a.headroom_gb << 30)) / (1 << 30))
    sc = SyntheticGRPOConfig(num_prompts=a.prompts_per_gpu * tp, prompt_len=a.prompt_len, group_size=a.group, temperature=1.0,
                             forced_len_median=a.median, forced_len_sigma=1.0, forced_len_min=16, forced_len_max=a.max_len,
                             eos_token_id=151645 % mcfg.vocab_size, merge_group_prompts=False, compute_ref_logprobs=not a.no_ref,
                             seed=1000 + dp_rank, use_cuda_graph=True, kv_gb=kv_gb, kv_memory_saver=True,
                             partial_rollout=not a.no_partial, inflight_prompts=a.inflight_per_gpu * tp, ref_on_device=ref_dev)
    pipe = SyntheticGRPO(mcfg, wc, grpo, sc, dev, train_engine=train)

    def barrier() -> None:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(a.warmup):
        st0 = dict(pipe.rollout.stats)
        m = pipe.run_step()
        if a.verbose and rank == 0:
            rs = {k: round(v - st0.get(k, 0), 3) for k, v in pipe.rollout.stats.items()}
            print(f"warmup {i}: " + json.dumps({k: round(v, 3) if isinstance(v, float) else v for k, v in m.items()
                                                 if k.endswith("_s") or k in ("trained_tokens", "loss", "grad_norm", "reward_mean")})
                  + " rollout " + json.dumps(rs), flush=True)

    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    _ext.count_launches(True, reset=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    start.record()
    tokens = 0
    step_metrics = []
    for _ in range(a.steps):
        m = pipe.run_step()  # public API: H2D of prompts/batches from pinned memory, D2H of loss/metrics
        tokens += m["trained_tokens"]
        step_metrics.append(m)
    end.record()
    barrier()
    wall = time.perf_counter() - wall0
    launches = _ext.count_launches(False)
    clk = clocks.stop()
    dev_ms = start.elapsed_time(end)

    phases = ("rollout_s", "logprob_s", "train_s", "sync_s", "pack_s")
    ph = [sum(m.get(k, 0.0) for m in step_metrics) / len(step_metrics) for k in phases]
    t = torch.tensor([dev_ms, wall, float(tokens), float(launches), *ph], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = t.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        dev_ms, wall = float(mx[0]), float(mx[1])
        tokens_all, launches_all = float(tot[2]) / tp, float(tot[3])  # the ranks of a TP group train the same tokens
        ph = [float(x) for x in mx[4:]]
    else:
        tokens_all, launches_all = float(tokens), float(launches)
    ms_step = dev_ms / a.steps
    value = tokens_all / (dev_ms / 1000.0)
    e2e = tokens_all / wall
    # bytes per step that the public API moves host<->device for this step's inputs/results
    last = step_metrics[-1]
    h2d = int(last.get("h2d_bytes", 0))
    d2h = int(last.get("d2h_bytes", 0))
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "trained tokens/s (whole job)",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": round(ms_step, 1),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random prompt ids, random-init weights, forced log-normal response lengths)",
            "config": {"model": f"{a.model} shape (36L, h4096, 32q/8kv, d128, ffn12288, vocab151936)" if a.model == "qwen3-8b" else a.model,
                       "global_batch": a.prompts_per_gpu * a.group * world, "prompts_per_step": a.prompts_per_gpu * world,
                       "group_size": a.group, "partial_rollout": not a.no_partial,
                       "inflight_groups": (a.inflight_per_gpu if not a.no_partial else a.prompts_per_gpu) * world,
                       "seq_len": a.prompt_len + a.max_len, "prompt_len": a.prompt_len,
                       "response_len": f"lognormal(median {a.median:g}, sigma 1) clipped [16,{a.max_len}]",
                       "micro_batch_tokens": a.mb_tokens, "parallelism": (f"tp{tp}" if tp > 1 else "") + f"dp{dp}" + (f"ep{ep}" if ep > 1 else ""), "colocated": True,
                       "ref_logprobs": not a.no_ref, "ref_weights": "device" if ref_dev else "pinned host", "deterministic_attention_backward": a.deterministic, "kv_pool_gb": round(kv_gb, 1), "l2": "inputs larger than L2 (weights 16 GB + KV cache per step)"},
            "sync_s": round(sum(m["sync_s"] for m in step_metrics) / len(step_metrics), 4),
            "step_breakdown_s": {k: round(v, 3) for k, v in zip(phases, ph)},
            "step_breakdown_note": "wall seconds per step, mean over the timed steps, max over ranks",
            "e2e": {"value": round(e2e, 1), "unit": "trained tokens/s (wall clock through SyntheticGRPO.run_step)",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches_all),
            "clocks": clk,
            "rollout_stats_per_step": {k: round(v / (a.warmup + a.steps), 3) for k, v in pipe.rollout.stats.items()},
        }
        print(json.dumps(out), flush=True)
    pipe.rollout.release_graphs()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Prefix-tree merged vs flat training forward+backward on multi-turn agentic trajectories.

Reference: ``benchmark/magi_forward/*.py`` (Magi merged-vs-THD forward sweeps) on the workload of
"multi-turn trajectories with prefix-tree packing": trajectories of 8-32 turns, each turn a
32-256-token action followed by a 64-512-token tool observation, context capped at 32768, groups
of 8 trajectories sharing a 2048-token prefix.  The flat layout trains every turn sample as its
own sequence (each re-reads its whole history); the merged layout packs each trajectory's trie
once (shared prefixes once, full-to-ancestors ranges).  Reports tokens processed, device time and
trained tokens per second for both.

python -m axrl_b200.benchmarks.merged_forward_bench [--model qwen3-8b] [--trajectories 8] [--layers N]
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def make_trajectories(n: int, rng: np.random.Generator, vocab: int, prefix: int = 2048, cap: int = 32768) -> list[list]:
    from axrl_b200.data.sample import Sample

    shared = rng.integers(1, vocab, size=prefix).tolist()
    trajs = []
    for _ in range(n):
        ctx = list(shared)
        turns = []
        for _t in range(int(rng.integers(8, 33))):
            act = rng.integers(1, vocab, size=int(rng.integers(32, 257))).tolist()
            if len(ctx) + len(act) > cap:
                break
            turns.append(Sample.from_tokens(list(ctx), act))
            obs = rng.integers(1, vocab, size=int(rng.integers(64, 513))).tolist()
            ctx = ctx + act + obs
            if len(ctx) >= cap:
                break
        trajs.append(turns)
    return trajs


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (memory)")
    ap.add_argument("--trajectories", type=int, default=4)
    ap.add_argument("--mb-tokens", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=2)
    a = ap.parse_args()
    from dataclasses import replace

    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.data.prefix_tree import merge_trajectory_samples
    from axrl_b200.data.sample import SampleBatch
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.train.engine import TrainEngine

    cfg = resolve_preset(a.model)
    if a.layers:
        cfg = replace(cfg, num_hidden_layers=a.layers)
    rng = np.random.default_rng(0)
    trajs = make_trajectories(a.trajectories, rng, cfg.vocab_size)
    eng = TrainEngine(MegatronWorkerConfig(inference_only=True, max_tokens_per_micro_batch=a.mb_tokens, recompute_granularity="full"),
                      cfg, "cuda")
    layouts = {"flat": [s for t in trajs for s in t], "merged": [merge_trajectory_samples(t, align_size=8) for t in trajs]}
    out = {"model": a.model, "layers": cfg.num_hidden_layers, "trajectories": len(trajs),
           "turn_samples": sum(len(t) for t in trajs)}
    for name, samples in layouts.items():
        batch = SampleBatch.from_samples(samples)
        tokens = int(sum(int(mb.num_tokens) for mb in eng.micro_batches(batch)))
        trained = int(batch["loss_mask"].sum())
        eng.model.train()
        for p in eng.model.parameters():
            p.requires_grad_(True)

        def step() -> None:
            for mb in eng.micro_batches(batch):
                d = mb.to("cuda")
                h = eng.model(d.ids, d.pos, d.spec)
                lp, _ = eng.model.logprobs(h, d.labels.clamp(min=-1))
                (lp * d.loss_mask).sum().backward()

        step()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            step()
        e.record()
        e.synchronize()
        sec = s.elapsed_time(e) / 1000 / a.iters
        out[name] = {"tokens_processed": tokens, "trained_tokens": trained, "seconds": round(sec, 3),
                     "trained_tokens_per_s": round(trained / sec, 1)}
    out["speedup_merged_vs_flat"] = round(out["flat"]["seconds"] / out["merged"]["seconds"], 2)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

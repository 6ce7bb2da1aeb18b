"""Multi-turn agentic GRPO benchmark on the Qwen3-8B shape (one GPU's share of the 64-trajectory step).

Trajectories of 8-32 turns (32-256-token model actions, 64-512-token tool observations of random
ids, context capped at 32768 tokens), in groups of 8 sharing a 2048-token prefix; partial rollout
carries unfinished groups across steps; training packs each finished group into prefix trees
(varlen block-mask attention over the tree ranges, loss on model tokens only).  Reference
counterpart: the agentic recipes' packed multi-turn training (``axrl/data/rollout_trace.py``,
``axrl/utils/megatron/prefix_tree.py``).  Reports device-timed (CUDA events) trained tokens/s
(packed tokens) and trajectory tokens/s (every context token of the trained trajectories).

python -m axrl_b200.benchmarks.agentic_bench [--steps 3] [--warmup 1] [--model qwen3-8b]
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--inflight-groups", type=int, default=2)
    ap.add_argument("--max-turns", type=int, default=32)
    ap.add_argument("--kv-gb", type=float, default=40.0)
    ap.add_argument("--mb-tokens", type=int, default=32768)
    a = ap.parse_args()
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.agentic_step import AgenticConfig, SyntheticAgentic
    from axrl_b200.train.engine import TrainEngine

    dev = torch.device("cuda", 0)
    mcfg = resolve_preset(a.model)
    wc = MegatronWorkerConfig(recompute_granularity="full", max_tokens_per_micro_batch=a.mb_tokens, deterministic_mode=False, seed=3)
    train = TrainEngine(wc, mcfg, dev)
    train.optim.release_grads()
    torch.cuda.empty_cache()
    ac = AgenticConfig(group_size=a.group, inflight_groups=a.inflight_groups, max_turns=a.max_turns, pack_len=a.mb_tokens, kv_gb=a.kv_gb,
                       eos_token_id=151645 % mcfg.vocab_size)
    pipe = SyntheticAgentic(mcfg, wc, GrpoTrainerConfig(loss_type="grpo"), ac, dev, train_engine=train)
    for _ in range(a.warmup):
        pipe.run_step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    start.record()
    ms = [pipe.run_step() for _ in range(a.steps)]
    end.record()
    torch.cuda.synchronize()
    dt = start.elapsed_time(end) / 1000.0
    packed = sum(m["trained_tokens"] for m in ms)
    logical = sum(m["trajectory_tokens"] for m in ms)
    print(json.dumps({"bench": "agentic_multi_turn", "model": a.model, "steps": a.steps, "s_per_step": round(dt / a.steps, 2),
                      "trained_tokens_per_s": round(packed / dt, 1), "trajectory_tokens_per_s": round(logical / dt, 1),
                      "wall_s": round(time.perf_counter() - wall0, 2),
                      "per_step": [{k: (round(v, 3) if isinstance(v, float) else v) for k, v in m.items()
                                    if k in ("rollout_s", "logprob_s", "train_s", "rounds", "turns", "trajectories", "trained_tokens",
                                             "trajectory_tokens", "generated_tokens", "carried_groups")} for m in ms]}), flush=True)
    pipe.rollout.release_graphs()


if __name__ == "__main__":
    main()

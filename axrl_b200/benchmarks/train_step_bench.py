"""Trainer-side GRPO phases on the dense GRPO workload, without the rollout.

The batch has the shape of one GRPO step of the dense benchmark: ``--prompts`` x ``--group``
sequences of a ``--prompt-len`` prompt followed by a response whose length is drawn log-normal
(median ``--median``, sigma 1, clipped to [16, ``--max-len``]), random token ids, random-init
weights.  Timed on the device with CUDA events:

* ``logprob``: one forward log-prob pass over the batch (the old- or reference-policy pass);
* ``train``: forward + backward of every packed micro-batch and the optimizer step.

``--one-micro-batch`` runs a single forward+backward of one micro-batch (for a kernel launch list).

Reference counterpart: the Megatron actor's ``compute_log_prob`` / ``update_policy``
(``axrl/worker/megatron_worker.py``), timed inside the reference's GRPO step.

python -m axrl_b200.benchmarks.train_step_bench [--prompts 32] [--group 8] [--mb-tokens 16384]
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def make_batch(n_prompts: int, group: int, prompt_len: int, median: float, max_len: int, vocab: int, seed: int = 0):  # noqa: ANN201
    from axrl_b200.data.sample import Sample, SampleBatch

    rng = np.random.default_rng(seed)
    samples = []
    for p in range(n_prompts):
        prompt = rng.integers(1, vocab, size=prompt_len).tolist()
        for _ in range(group):
            n = int(np.clip(np.exp(np.log(median) + rng.standard_normal()), 16, max_len))
            resp = rng.integers(1, vocab, size=n).tolist()
            lp = (-rng.random(n) * 4).astype(np.float32)
            samples.append(Sample.from_tokens(prompt, resp, reward=float(rng.random() < 0.5), advantage=float(rng.standard_normal()),
                                              rollout_logprobs=lp, trajectory_id=p))
    return SampleBatch.from_samples(samples)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--median", type=float, default=1024.0)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--mb-tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--one-micro-batch", action="store_true")
    ap.add_argument("--deterministic", action="store_true", help="deterministic attention backward (separate dQ pass), as bench.py --deterministic")
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args()

    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.train.engine import TrainEngine
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer

    cfg = resolve_preset(a.model)
    dev = torch.device(a.device)
    cuda = dev.type == "cuda"
    eng = TrainEngine(MegatronWorkerConfig(recompute_granularity="full", max_tokens_per_micro_batch=a.mb_tokens, seed=1234,
                                           deterministic_mode=a.deterministic), cfg, dev)
    trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo", mismatch_token_clip_max=2.0))
    batch = make_batch(a.prompts, a.group, a.prompt_len, a.median, a.max_len, cfg.vocab_size)
    tokens = int(batch["seq_len"].sum())

    if a.one_micro_batch:
        mb = eng.micro_batches(batch)[0]
        eng.model.train()
        for _ in range(a.iters):
            d = mb.to(dev)
            h = eng._hidden(d)
            lp, _ = eng.model.logprobs(h, d.labels.clamp(min=-1), 1.0)
            (lp.float() * (d.labels >= 0)).sum().backward()
            eng.optim.zero_grad()
        if cuda:
            torch.cuda.synchronize()
        print(json.dumps({"micro_batch_tokens": int(mb.num_tokens), "iters": a.iters}))
        return

    def timed(fn) -> float:  # noqa: ANN001
        if not cuda:
            import time

            t0 = time.perf_counter()
            fn()
            return time.perf_counter() - t0
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / 1000.0

    def logprob() -> None:
        batch["old_logprobs"] = eng.compute_logprobs(batch, 1.0)

    out = {"model": a.model, "sequences": a.prompts * a.group, "tokens": tokens, "micro_batches": len(eng.micro_batches(batch))}
    lp_s, tr_s = [], []
    for _ in range(a.iters):
        lp_s.append(timed(logprob))
        batch["ref_logprobs"] = batch["old_logprobs"]
        tr_s.append(timed(lambda: eng.train_step(batch, trainer, metrics_every_micro_batch=False)))
    lp, tr = min(lp_s), min(tr_s)
    out.update({"logprob_s": round(lp, 3), "train_s": round(tr, 3), "logprob_tok_s": round(tokens / lp, 1),
                "train_tok_s": round(tokens / tr, 1)})
    print(json.dumps(out))


if __name__ == "__main__":
    main()

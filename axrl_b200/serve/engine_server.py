"""One rollout engine served over HTTP (``/generate`` with token ids; input-logprob scoring for
OPD teachers).

Reference: the standalone SGLang servers the reference launches for teachers
(``axrl/utils/sglang_launch_utils.py:222-286``).  Usage:

``python -m axrl_b200.serve.engine_server --preset qwen3-8b --port 30000 [--device cuda:0] [--hf-dir DIR]``
"""

from __future__ import annotations

import argparse

import numpy as np
import torch


def build_worker(preset: str, device: str, hf_dir: str | None, max_batch: int, max_context: int, seed: int):  # noqa: ANN201
    from axrl_b200.configs import SamplingConfig
    from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
    from axrl_b200.rollout.engine import RolloutEngine
    from axrl_b200.worker.rollout_worker import RolloutWorker

    dtype = torch.bfloat16 if device.startswith("cuda") else torch.float32
    if hf_dir:  # a Hugging Face Qwen3 checkpoint directory (config.json + safetensors)
        from axrl_b200.train.checkpoint import hf_config, load_hf_checkpoint

        cfg = hf_config(hf_dir)
        model = Qwen3Model(cfg)
        load_hf_checkpoint(model, hf_dir)
    else:
        cfg = resolve_preset(preset)
        model = Qwen3Model(cfg)
        model.init_weights(seed)
    model = model.to(device=device, dtype=dtype)
    model.inv_freq = model.inv_freq.float()
    for p in model.parameters():
        p.requires_grad_(False)
    engine = RolloutEngine(model, max_batch=max_batch, kv_tokens=max_batch * max_context, max_context=max_context, seed=seed,
                           use_cuda_graph=device.startswith("cuda"))
    worker = RolloutWorker(engine, SamplingConfig())

    @torch.no_grad()
    def teacher(ids: np.ndarray, start: int) -> list:
        from axrl_b200.ops.attention_spec import spec_from_triples

        n = len(ids)
        spec = spec_from_triples([(0, n, 0, n, 1)], n)
        if device.startswith("cuda"):
            spec = spec.to(device)
        t = torch.as_tensor(ids, device=device).long()
        h = model(t, torch.arange(n, device=device, dtype=torch.int32), spec)
        labels = torch.cat([t[1:], t.new_full((1,), -1)])
        lp, _ = model.logprobs(h, labels)
        vals = lp.float().cpu().tolist()
        return [[None if i < start else float(vals[i - 1]), int(ids[i]), None] for i in range(start, n)]

    return worker, teacher


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--hf-dir", default=None)
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-context", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    import uvicorn

    from axrl_b200.worker.oai_client import create_generate_app

    worker, teacher = build_worker(a.preset, a.device, a.hf_dir, a.max_batch, a.max_context, a.seed)
    uvicorn.run(create_generate_app(worker, teacher_model=teacher), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()

"""Expert-parallel rollout for MoE models on CPU: two gloo ranks, each holding half the experts and
running the same requests (attention replicated, expert FFNs dispatched to their owners), produce
the same tokens and log-probs as a single engine over the full model (reference counterpart: SGLang
engines with ``ep_size``, ``axrl/configs.py:210-214``)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reqs():
    from axrl_b200.rollout.engine import GenRequest

    g = torch.Generator().manual_seed(3)
    return [GenRequest(rid=f"r{i}", prompt=torch.randint(1, 1024, (n,), generator=g).tolist(), max_new_tokens=10, temperature=1.0,
                       seed_stream=i) for i, n in enumerate((7, 12, 9))]


def _worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
        from axrl_b200.parallel.expert import EPContext, load_ep_shards_from_full
        from axrl_b200.rollout.engine import RolloutEngine

        cfg = resolve_preset("tiny-moe")
        full = Qwen3Model(cfg)
        full.init_weights(2)
        ref = RolloutEngine(full, max_batch=4, kv_tokens=2048, max_context=128, use_cuda_graph=False, seed=4).generate(_reqs())
        ep = EPContext.from_group(dist.group.WORLD)
        model = Qwen3Model(cfg, ep=ep)
        load_ep_shards_from_full(model, {k: v.detach() for k, v in full.named_parameters()}, ep)
        assert model.layers[0].mlp.experts_gate_up.shape[0] == cfg.num_experts // world
        got = RolloutEngine(model, max_batch=4, kv_tokens=2048, max_context=128, use_cuda_graph=False, seed=4).generate(_reqs())
        for a, b in zip(got, ref):
            assert a.output_ids == b.output_ids, (a.output_ids, b.output_ids)
            torch.testing.assert_close(torch.tensor(a.output_logprobs), torch.tensor(b.output_logprobs), atol=1e-4, rtol=1e-4)
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_ep2_rollout_matches_single_engine():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def _dp_reqs(rank: int):
    from axrl_b200.rollout.engine import GenRequest

    g = torch.Generator().manual_seed(11 + rank)
    lens, news = ((7, 12, 9), (10, 4, 14)) if rank == 0 else ((5, 16), (3, 9))  # ranks finish at different steps
    return [GenRequest(rid=f"d{rank}_{i}", prompt=torch.randint(1, 1024, (n,), generator=g).tolist(), max_new_tokens=m,
                       temperature=1.0, seed_stream=100 * rank + i) for i, (n, m) in enumerate(zip(lens, news))]


def _dp_worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
        from axrl_b200.parallel.expert import EPContext, load_ep_shards_from_full
        from axrl_b200.rollout.engine import RolloutEngine

        cfg = resolve_preset("tiny-moe")
        full = Qwen3Model(cfg)
        full.init_weights(2)
        ref = RolloutEngine(full, max_batch=4, kv_tokens=2048, max_context=128, use_cuda_graph=False, seed=4, burst=4).generate(_dp_reqs(rank))
        ep = EPContext.from_group(dist.group.WORLD)
        model = Qwen3Model(cfg, ep=ep)
        load_ep_shards_from_full(model, {k: v.detach() for k, v in full.named_parameters()}, ep)
        eng = RolloutEngine(model, max_batch=4, kv_tokens=2048, max_context=128, seed=4, burst=4, dp_attention=True)
        got = eng.generate(_dp_reqs(rank))
        for a, b in zip(got, ref):
            assert a.output_ids == b.output_ids, (a.output_ids, b.output_ids)
            torch.testing.assert_close(torch.tensor(a.output_logprobs), torch.tensor(b.output_logprobs), atol=1e-4, rtol=1e-4)
        # a rank with no requests still joins the other ranks' forwards
        extra = _dp_reqs(0)[:1] if rank == 0 else []
        got2 = eng.generate(extra)
        assert len(got2) == len(extra) and all(len(r.output_ids) == 10 for r in got2)
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_ep2_dp_attention_rollout_matches_single_engines():
    """Data-parallel attention: each EP rank serves different requests (attention and KV cache per
    rank, experts shared through the EP dispatch); results equal one engine per request set."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def _worker_lockstep(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import asyncio

        import numpy as np

        from axrl_b200.configs import SamplingConfig
        from axrl_b200.data.conversation import GenerationInput
        from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
        from axrl_b200.parallel.expert import EPContext
        from axrl_b200.rollout.engine import RolloutEngine
        from axrl_b200.worker.rollout_worker import RolloutWorker

        cfg = resolve_preset("tiny-moe")
        model = Qwen3Model(cfg, ep=EPContext.from_group(dist.group.WORLD))
        model.init_weights(2)
        eng = RolloutEngine(model, max_batch=4, kv_tokens=2048, max_context=128, seed=4, burst=4, dp_attention=True)
        w = RolloutWorker(eng, SamplingConfig(max_new_tokens=6 + 5 * rank, temperature=1.0))
        g = np.random.default_rng(rank)

        async def batch(n: int) -> list:
            return await asyncio.gather(*[w.generate(GenerationInput(session_id=f"s{rank}_{i}", input_ids=g.integers(1, 1024, 9 + i)))
                                          for i in range(n)])

        outs = asyncio.run(batch(2 + rank))
        assert all(len(o.output_ids) == 6 + 5 * rank for o in outs)
        w.pause_generation()  # both ranks: the engine threads pause together
        dist.barrier()  # stands in for training collectives between pause and resume
        w.resume_generation()
        outs = asyncio.run(batch(1))
        assert len(outs[0].output_ids) == 6 + 5 * rank
        # A stop from any rank ends every rank's engine loop, so shut down once every rank is done:
        # pause first (no expert collectives in flight), then meet, then stop.
        w.pause_generation()
        dist.barrier()
        w.shutdown()
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_rollout_worker_lockstep_with_dp_attention():
    """Rollout workers over data-parallel-attention engines: per-rank requests of different lengths,
    a pause / resume between them, and shutdown, with the engine threads in lockstep."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_lockstep, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def _worker_one_rank_stops(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import asyncio

        import numpy as np

        from axrl_b200.configs import SamplingConfig
        from axrl_b200.data.conversation import GenerationInput
        from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
        from axrl_b200.parallel.expert import EPContext
        from axrl_b200.rollout.engine import RolloutEngine
        from axrl_b200.worker.rollout_worker import RolloutWorker

        cfg = resolve_preset("tiny-moe")
        model = Qwen3Model(cfg, ep=EPContext.from_group(dist.group.WORLD))
        model.init_weights(2)
        eng = RolloutEngine(model, max_batch=4, kv_tokens=4096, max_context=512, seed=4, burst=4, dp_attention=True)
        budget = 400 if rank == 0 else 4
        w = RolloutWorker(eng, SamplingConfig(max_new_tokens=budget, temperature=1.0))
        g = np.random.default_rng(rank)

        async def run() -> list:
            calls = [w.generate(GenerationInput(session_id=f"s{rank}_{i}", input_ids=g.integers(1, 1024, 9 + i))) for i in range(3)]
            if rank == 0:
                return await asyncio.gather(*calls)
            outs = await asyncio.gather(*calls)
            w.shutdown()  # only this rank asks; rank 0 still has requests in flight
            return outs

        outs = asyncio.run(asyncio.wait_for(run(), timeout=120))
        w._thread.join(timeout=30)
        assert not w._thread.is_alive(), "engine thread still running"
        if rank == 0:
            assert all(o.finish_reason == "abort" or len(o.output_ids) == budget for o in outs), [o.finish_reason for o in outs]
            assert any(o.finish_reason == "abort" for o in outs)
            # a call after the stop resolves at once instead of waiting for an engine that is gone
            late = asyncio.run(asyncio.wait_for(w.generate(GenerationInput(session_id="late", input_ids=np.arange(1, 9))), timeout=10))
            assert late.finish_reason == "abort" and len(late.output_ids) == 0
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_rollout_worker_lockstep_stop_on_one_rank_resolves_all_calls():
    """One rank shuts its worker down while the other still generates: both engine threads stop at
    the same decision, the busy rank's calls return their partial output as aborted, and a call made
    after the stop resolves immediately."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_one_rank_stops, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"

"""Pipeline parallelism on CPU: two gloo ranks (PP=2, 1F1B) against the PP=1 engine on the same
batch — logprob recompute, GRPO loss, grad norm and the updated parameters (Megatron's
non-interleaved schedule, ``axrl/worker/megatron_worker.py:950-1031``)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch():
    from axrl_b200.data.sample import Sample, SampleBatch

    g = torch.Generator().manual_seed(4)
    samples = []
    for i in range(7):
        n_p, n_r = 5 + i, 6 + 2 * i
        p = torch.randint(1, 200, (n_p,), generator=g).tolist()
        r = torch.randint(1, 200, (n_r,), generator=g).tolist()
        lp = (-torch.rand(n_r, generator=g)).tolist()
        samples.append(Sample.from_tokens(p, r, reward=float(i % 2), advantage=float(i % 3) - 1.0, rollout_logprobs=lp,
                                          trajectory_id=i))
    return SampleBatch.from_samples(samples)


def _engine(par=None):
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.models.qwen3 import Qwen3Config
    from axrl_b200.train.engine import TrainEngine

    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=5, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16)
    wc = MegatronWorkerConfig(max_tokens_per_micro_batch=40, seed=7)
    wc.lr_scheduler.lr_warmup_steps = 0
    wc.lr_scheduler.max_lr = 1e-3
    return TrainEngine(wc, cfg, "cpu", par=par)


def _worker(rank: int, world: int, port: int, q, vpp: int = 1) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.configs import GrpoTrainerConfig
        from axrl_b200.train.engine import ParallelCtx
        from axrl_b200.trainer.grpo_trainer import GrpoTrainer

        ref = _engine()
        eng = _engine(ParallelCtx(pp_group=dist.group.WORLD, pp_size=world, vpp_size=vpp))
        if vpp == 1:
            assert len(eng.model.layers) in (2, 3) and eng.model.layer_offset == (0 if rank == 0 else 3)
        else:  # 5 layers over 4 virtual stages: rank 0 holds layers 0-1 and 3, rank 1 layers 2 and 4
            offs = [ch.layer_offset for ch in eng.model.chunks]
            assert offs == ([0, 3] if rank == 0 else [2, 4]), offs
        b = _batch()
        assert len(eng.micro_batches(b)) >= 3  # warm-up, steady state and cool-down all run
        lp_ref = ref.compute_logprobs(b)
        lp = eng.compute_logprobs(b)
        torch.testing.assert_close(lp, lp_ref, atol=1e-5, rtol=1e-5)
        b["old_logprobs"] = lp_ref
        b["ref_logprobs"] = lp_ref
        trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo"))
        m_ref = ref.train_step(b, trainer)
        m = eng.train_step(b, trainer)
        assert abs(m["grad_norm"] - m_ref["grad_norm"]) < 1e-4 * max(1.0, m_ref["grad_norm"]), (m["grad_norm"], m_ref["grad_norm"])
        assert abs(m["loss"] - m_ref["loss"]) < 1e-5
        refp = {n: p for n, p in ref.model.named_parameters()}
        for n, p in eng.model.named_parameters():
            torch.testing.assert_close(p, refp[eng.model.global_name(n)], atol=1e-6, rtol=1e-5)
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_pp2_1f1b_matches_pp1():
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


def test_pp2_interleaved_vpp2_matches_pp1():
    """Two virtual stages per rank (interleaved 1F1B, Megatron ``virtual_pipeline_model_parallel_size``):
    the activation walks both ranks twice; results must equal the PP=1 engine."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, 2)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def test_interleaved_plan_is_complete_and_deadlock_free():
    from axrl_b200.parallel.pipeline import interleaved_order, plan_interleaved

    for P in (2, 3, 4, 8):
        for V in (1, 2, 3, 4):
            for n in range(1, 20):
                plan = plan_interleaved(P, V, n)
                for r in range(P):
                    acts = [a[r] for a in plan.actions if a[r] is not None]
                    assert sorted(acts) == sorted(interleaved_order(P, V, r, n))
                    # a backward never precedes its own forward on a rank
                    seen = set()
                    for kind, mb, c in acts:
                        if kind == "F":
                            seen.add((mb, c))
                        else:
                            assert (mb, c) in seen
    # interleaving shortens the pipeline (ticks weighted by chunk size)
    assert len(plan_interleaved(4, 2, 8).actions) / 2 < len(plan_interleaved(4, 1, 8).actions)


def test_layer_ranges():
    from axrl_b200.parallel.pipeline import PPContext

    ranges = [PPContext(size=4, rank=r, ranks=[0, 1, 2, 3]).layer_range(10) for r in range(4)]
    assert ranges == [(0, 3), (3, 6), (6, 8), (8, 10)]

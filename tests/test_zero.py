"""Bucketed ZeRO-1 AdamW (reduce-scatter per bucket, sharded Adam, parameter gather) on two gloo
ranks against the replicated optimizer with a full gradient all-reduce (Megatron distributed
optimizer, ``axrl/worker/megatron_worker.py:905-930``)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
        from axrl_b200.models.qwen3 import Qwen3Config
        from axrl_b200.parallel.zero import BucketedZeroAdamW
        from axrl_b200.train.engine import ParallelCtx, TrainEngine
        from axrl_b200.trainer.grpo_trainer import GrpoTrainer
        from tests.test_pipeline_parallel import _batch

        cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=4,
                          num_key_value_heads=2, head_dim=16)

        def engine(zero: str):
            wc = MegatronWorkerConfig(max_tokens_per_micro_batch=48, seed=5)
            wc.lr_scheduler.lr_warmup_steps = 0
            wc.lr_scheduler.max_lr = 1e-3
            return TrainEngine(wc, cfg, "cpu", par=ParallelCtx(dp_group=dist.group.WORLD, dp_size=world, zero_backend=zero))

        ref, eng = engine("off"), engine("nccl")
        assert isinstance(eng.optim, BucketedZeroAdamW) and len(eng.optim.buckets) >= 2
        b = _batch()
        rows = [i for i in range(len(b)) if i % world == rank]  # each DP rank trains its own rows
        b = b.select_rows(rows)
        lp = ref.compute_logprobs(b)
        b["old_logprobs"] = lp
        b["ref_logprobs"] = lp
        trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo"))
        for _ in range(2):
            m_ref = ref.train_step(b, trainer)
            m = eng.train_step(b, trainer)
            assert abs(m["grad_norm"] - m_ref["grad_norm"]) < 1e-4 * max(1.0, m_ref["grad_norm"]), (m["grad_norm"], m_ref["grad_norm"])
        for (n, p), pr in zip(eng.model.named_parameters(), ref.model.parameters()):
            torch.testing.assert_close(p, pr, atol=1e-6, rtol=1e-5, msg=lambda msg, n=n: f"{n}: {msg}")
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_bucketed_zero_matches_replicated_adam():
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


def test_backward_order_groups():
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.parallel.zero import backward_order_groups

    m = Qwen3Model(Qwen3Config(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=3, num_attention_heads=2,
                               num_key_value_heads=1, head_dim=16))
    g = backward_order_groups(m)
    assert [t for t, _ in g] == [2, 1, 0, None]
    assert g[0][1][0] is m.norm.weight and g[-1][1] == [m.embed_tokens]
    assert sum(len(ps) for _, ps in g) == len(list(m.parameters()))

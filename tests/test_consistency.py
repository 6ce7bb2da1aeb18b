"""Cross-rank consistency checks (replicated tensors compared by checksum across gloo ranks), and the
trainer's per-step check of data-parallel replicas."""

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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AXRL_CONSISTENCY_CHECKS="1")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
        from axrl_b200.models.qwen3 import Qwen3Config
        from axrl_b200.train.engine import ParallelCtx, TrainEngine
        from axrl_b200.trainer.grpo_trainer import GrpoTrainer
        from axrl_b200.utils.consistency import check_replicated
        from tests.test_pipeline_parallel import _batch

        a = torch.arange(10.0)
        check_replicated([("a", a)])  # identical: passes
        try:
            check_replicated([("a", a), ("b", a + rank)])
            raise AssertionError("divergence not detected")
        except RuntimeError as e:
            assert "['b']" in str(e), str(e)
        cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                          num_key_value_heads=2, head_dim=16)
        wc = MegatronWorkerConfig(max_tokens_per_micro_batch=64, seed=5)
        eng = TrainEngine(wc, cfg, "cpu", par=ParallelCtx(dp_group=dist.group.WORLD, dp_size=world, zero_backend="off"))
        b = _batch()
        b = b.select_rows([i for i in range(len(b)) if i % world == rank])
        lp = eng.compute_logprobs(b)
        b["old_logprobs"] = lp
        b["ref_logprobs"] = lp
        eng.train_step(b, GrpoTrainer(GrpoTrainerConfig(loss_type="grpo")))  # checked inside: replicas agree
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_replica_checks_detect_divergence_and_pass_after_a_step():
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

"""Expert parallelism on CPU: two gloo ranks (EP=2), each with its own tokens, against the EP=1
model on the same tokens (Megatron alltoall dispatcher semantics,
``axrl/worker/megatron_worker.py:833``)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q, etp: int = 1) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.models.moe import MoEContext
        from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
        from axrl_b200.ops.attention_spec import spec_from_triples
        from axrl_b200.parallel.expert import EPContext, expert_params, load_ep_shards_from_full

        cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                          num_key_value_heads=2, head_dim=16, num_experts=8, num_experts_per_tok=3, moe_intermediate_size=32)
        full = Qwen3Model(cfg)
        full.init_weights(11)
        state = {k: v.detach().clone() for k, v in full.named_parameters()}
        if etp == 1:
            ep = EPContext.from_group(dist.group.WORLD)
        else:  # ETP groups {0,1},{2,3}; EP groups {0,2},{1,3} (every rank belongs to one of each)
            ep_groups = [dist.new_group([r for r in range(world) if r % etp == i]) for i in range(etp)]
            etp_groups = [dist.new_group(list(range(e * etp, (e + 1) * etp))) for e in range(world // etp)]
            ep = EPContext.from_group(ep_groups[rank % etp], etp_group=etp_groups[rank // etp])
        model = Qwen3Model(cfg, ep=ep)
        load_ep_shards_from_full(model, state, ep)
        ep_size = world // etp
        assert model.layers[0].mlp.experts_gate_up.shape == (8 // ep_size, 2 * 32 // etp, 64)

        T = 20 + 6 * rank  # different token counts per rank
        g = torch.Generator().manual_seed(100 + rank)
        ids = torch.randint(0, 256, (T,), generator=g)
        labels = torch.randint(0, 256, (T,), generator=g)
        spec = spec_from_triples([(0, T, 0, T, 1)], T)
        pos = torch.arange(T).int()
        # replay: layer 1 uses recorded experts for the first half of the tokens
        rep = torch.randint(0, 8, (T, 3), generator=g)
        for j in range(3):  # distinct experts per token
            rep[:, j] = (rep[:, 0] + j) % 8
        mask = torch.arange(T) < T // 2

        def run(m):
            for p in m.parameters():
                p.main_grad = torch.zeros(p.shape)
                p.grad = None
            ctx = MoEContext(replay={1: rep}, replay_mask=mask)
            h = m(ids, pos, spec, ctx)
            lp, _ = m.logprobs(h, labels)
            lp.sum().backward()
            for p in m.parameters():
                if p.grad is not None:
                    p.main_grad += p.grad
                    p.grad = None
            return lp.detach()

        lp_ref = run(full)
        lp = run(model)
        torch.testing.assert_close(lp, lp_ref, atol=1e-4, rtol=1e-4)
        fulld = dict(full.named_parameters())
        for n, p in model.named_parameters():
            ref = fulld[n].main_grad
            if getattr(p, "expert_parallel", False):
                ref = ref.clone()
                dist.all_reduce(ref)  # every rank's tokens reach the owner's experts
                E_l = p.shape[0]
                ref = ref[ep.rank * E_l:(ep.rank + 1) * E_l]
                if etp > 1:  # this rank's FFN columns
                    r = ep.etp_rank
                    if n.endswith("experts_gate_up"):
                        F, Fl = ref.shape[1] // 2, p.shape[1] // 2
                        ref = torch.cat([ref[:, r * Fl:(r + 1) * Fl], ref[:, F + r * Fl:F + (r + 1) * Fl]], 1)
                    else:
                        Fl = p.shape[2]
                        ref = ref[:, :, r * Fl:(r + 1) * Fl]
            torch.testing.assert_close(p.main_grad, ref, atol=1e-4, rtol=1e-3, msg=lambda m, n=n: f"{n}: {m}")
        assert len(expert_params(model)) == 2 * cfg.num_hidden_layers
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_ep2_matches_ep1_with_replay():
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


def test_ep2_x_etp2_matches_ep1():
    """Expert tensor parallelism (Megatron ``expert_tensor_parallel_size``, ``axrl/configs.py:384``):
    4 ranks = EP 2 x ETP 2; each expert's FFN columns split over an ETP pair, rows all-gathered
    before and partial sums reduce-scattered after the expert FFN."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 4, port, q, 2)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def test_grouped_linear_cpu_matches_loop():
    from axrl_b200.ops.grouped import expert_offsets, grouped_linear

    ids = torch.tensor([0, 0, 2, 2, 2, 3])
    off = expert_offsets(ids, 5)
    assert off.tolist() == [0, 2, 2, 5, 6, 6]
    x = torch.randn(6, 8)
    w = torch.randn(5, 4, 8)
    y = grouped_linear(x, w, off)
    torch.testing.assert_close(y[2:5], x[2:5] @ w[2].t())

"""Context parallelism on CPU: gloo ranks (zigzag split, ring attention over the per-source key
chunks, or the all-gathered keys/values) against the CP=1 engine on the same batch, flat sequences plus a prefix-tree merged group
(``axrl/utils/megatron/pack_utils.py:35-36,91-106``)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(tree: bool = True):
    from axrl_b200.data.prefix_tree import merge_trajectory_samples
    from axrl_b200.data.sample import Sample, SampleBatch

    g = torch.Generator().manual_seed(9)
    samples = []
    for i in range(4):
        p = torch.randint(1, 200, (7 + 3 * i,), generator=g).tolist()
        r = torch.randint(1, 200, (9 + 5 * i,), generator=g).tolist()
        samples.append(Sample.from_tokens(p, r, advantage=float(i % 3) - 1.0, rollout_logprobs=(-torch.rand(len(r), generator=g)).tolist(),
                                          trajectory_id=i))
    if not tree:
        return SampleBatch.from_samples(samples)
    prompt = torch.randint(1, 200, (11,), generator=g).tolist()
    group = []
    for j in range(3):
        r = torch.randint(1, 200, (6 + 4 * j,), generator=g).tolist()
        group.append(Sample.from_tokens(prompt, r, advantage=1.0 - j, rollout_logprobs=(-torch.rand(len(r), generator=g)).tolist(),
                                        trajectory_id=10))
    samples.append(merge_trajectory_samples(group, align_size=1))
    return SampleBatch.from_samples(samples)


def _engine(par=None, hybrid: bool = False):
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.models.qwen3 import Qwen3Config
    from axrl_b200.train.engine import TrainEngine

    kw = {}
    if hybrid:  # a Gated DeltaNet layer (heads exchanged for tokens by all-to-all) + gated attention
        kw = dict(layer_types=["linear_attention", "full_attention"], linear_num_key_heads=2, linear_num_value_heads=4,
                  linear_key_head_dim=16, linear_value_head_dim=8, attn_output_gate=True, partial_rotary_factor=0.5)
    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, **kw)
    wc = MegatronWorkerConfig(max_tokens_per_micro_batch=48, seed=3)
    wc.lr_scheduler.lr_warmup_steps = 0
    wc.lr_scheduler.max_lr = 1e-3
    return TrainEngine(wc, cfg, "cpu", par=par)


def _worker(rank: int, world: int, port: int, q, hybrid: bool = False, cp_attn: str = "ring") -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AXRL_CP_ATTN=cp_attn)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.configs import GrpoTrainerConfig
        from axrl_b200.train.engine import ParallelCtx
        from axrl_b200.trainer.grpo_trainer import GrpoTrainer

        ref = _engine(hybrid=hybrid)
        eng = _engine(ParallelCtx(cp_group=dist.group.WORLD, cp_size=world), hybrid=hybrid)
        b = _batch(tree=not hybrid)
        lp_ref = ref.compute_logprobs(b)
        lp = eng.compute_logprobs(b)
        torch.testing.assert_close(lp, lp_ref, atol=1e-5, rtol=1e-5)
        b["old_logprobs"] = lp_ref
        b["ref_logprobs"] = lp_ref
        trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo", loss_agg_type="token-mean"))
        m_ref = ref.train_step(b, trainer)
        m = eng.train_step(b, trainer)
        assert abs(m["grad_norm"] - m_ref["grad_norm"]) < 1e-4 * max(1.0, m_ref["grad_norm"]), (m["grad_norm"], m_ref["grad_norm"])
        # Adam normalises each element's gradient, so near-zero gradients summed in another order
        # (the ring's per-source attention backward, the GDN all-to-all path) can move an element
        # by a fraction of one lr-sized step
        atol = 2e-5
        for (n, p), pr in zip(eng.model.named_parameters(), ref.model.parameters()):
            torch.testing.assert_close(p, pr, atol=atol, rtol=1e-5, msg=lambda msg, n=n: f"{n}: {msg}")
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,hybrid,cp_attn", [(2, False, "ring"), (2, True, "ring"), (2, False, "gather"), (3, False, "ring")])
def test_cp_matches_cp1(world, hybrid, cp_attn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, hybrid, cp_attn)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


def test_zigzag_spec_covers_causal_mask():
    """Gathered-key spec of both ranks reproduces the causal mask of one long row."""
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.ops.attention_spec import dense_mask
    from axrl_b200.parallel.context_parallel import CPContext, pack_rows_cp

    b = SampleBatch.from_samples([Sample.from_tokens(list(range(1, 14)), list(range(20, 31)))])
    n = 24
    full = torch.tril(torch.ones(n, n, dtype=torch.bool))
    rows = []
    for r in range(2):
        mb = pack_rows_cp(b, [0], CPContext(size=2, rank=r))
        m = dense_mask(mb.spec)  # (L, 2L) over rank-major gathered keys
        L = mb.num_tokens
        cols = torch.cat([pack_rows_cp(b, [0], CPContext(size=2, rank=k)).token_col for k in range(2)])
        valid_k = torch.cat([pack_rows_cp(b, [0], CPContext(size=2, rank=k)).token_row >= 0 for k in range(2)])
        for i in range(L):
            if mb.token_row[i] < 0:
                continue
            qi = int(mb.token_col[i])
            got = {int(cols[j]) for j in range(2 * L) if m[i, j] and valid_k[j]}
            assert got == {j for j in range(n) if full[qi, j]}, (r, qi)
        rows.append(L)
    assert rows[0] == rows[1]


def test_split_key_attention_matches_full():
    """Per-source partials merged by log-sum-exp, and the per-source backward against the final
    (o, lse), equal full attention and its autograd gradients (keys split over three sources)."""
    from axrl_b200.ops import core as ops
    from axrl_b200.ops.attention_spec import spec_from_triples

    torch.manual_seed(0)
    T, S, Hq, Hkv, D = 12, 3, 4, 2, 16
    scale = D ** -0.5
    triples = [(0, 12, 0, 8, 0), (0, 12, 8, 20, 1), (4, 12, 20, 30, 0)]  # full, causal, partial-row full
    q = torch.randn(T, Hq, D, dtype=torch.float64, requires_grad=True)
    k = torch.randn(30, Hkv, D, dtype=torch.float64, requires_grad=True)
    v = torch.randn(30, Hkv, D, dtype=torch.float64, requires_grad=True)
    full = spec_from_triples(triples, T, 30)
    o_ref = ops._attn_ref(q, k, v, full, scale)
    do = torch.randn_like(o_ref)
    o_ref.backward(do)
    bounds = [(0, 10), (10, 20), (20, 30)]
    srcs = []
    for a, b in bounds:
        tr = []
        for q0, q1, k0, k1, t in triples:
            ka, kb = max(k0, a), min(k1, b)
            qa = q0 + (ka - k0) if t == 1 else q0  # a causal range cut at ka starts ka-k0 queries later
            if ka < kb and qa < q1:
                tr.append((qa, q1, ka - a, kb - a, t))
        srcs.append(spec_from_triples(tr, T, b - a))
    qd, kd, vd = q.detach(), k.detach(), v.detach()
    parts = [ops.attn_partial(qd, kd[a:b], vd[a:b], sp, scale) for (a, b), sp in zip(bounds, srcs)]
    o, lse2 = ops.attn_merge(parts)
    torch.testing.assert_close(o, o_ref.detach(), atol=1e-5, rtol=1e-5)  # the partials compute in fp32
    dsum = ops.attn_bwd_dsum(o, do)
    dq = torch.zeros(q.shape, dtype=torch.float32)
    dks, dvs = [], []
    for (a, b), sp in zip(bounds, srcs):
        dk, dv = ops.attn_bwd_partial(do, qd, kd[a:b], vd[a:b], lse2, dsum, dq, sp, scale)
        dks.append(dk)
        dvs.append(dv)
    torch.testing.assert_close(dq.double(), q.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(torch.cat(dks), k.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(torch.cat(dvs), v.grad, atol=1e-5, rtol=1e-5)

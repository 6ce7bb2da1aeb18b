"""Host runtime (native block manager vs Python twin), micro-batch balancing, and the
tiny CPU GRPO plumbing run (2 layers, hidden 256, 4 heads, FFN 768, vocab 1024, fp32)."""

import numpy as np
import torch

from axrl_b200.rollout.kv import PyBlockManager, make_block_manager
from axrl_b200.train.packing import split_balanced


def test_block_manager_native_matches_python():
    rng = np.random.default_rng(0)
    nat = make_block_manager(32, 4)
    py = PyBlockManager(32, 4)
    assert type(nat).__name__ == "BlockManager", "native runtime module not loaded"
    owned = []
    for it in range(300):
        op = rng.integers(0, 4)
        if op == 0 and nat.num_available() > 3:
            a, b = nat.allocate(3), py.allocate(3)
            assert a == b
            owned.append(a)
        elif op == 1 and owned:
            pages = owned.pop(int(rng.integers(0, len(owned))))
            nat.release(pages)
            py.release(pages)
        elif op == 2 and owned:
            toks = rng.integers(0, 5, size=12).tolist()
            pages = owned[-1]
            nat.insert(toks, pages)
            py.insert(toks, pages)
        else:
            toks = rng.integers(0, 5, size=12).tolist()
            ma, mb = nat.match_prefix(toks), py.match_prefix(toks)
            assert list(ma[0]) == list(mb[0]) and ma[1] == mb[1]
            if ma[0]:
                owned.append(list(ma[0]))
        assert nat.num_available() == py.num_available()
        assert nat.num_free() == py.num_free()


def test_prefix_cache_reuse_and_eviction():
    bm = make_block_manager(4, 2)
    t = [1, 2, 3, 4]
    p = bm.allocate(2)
    bm.insert(t, p)
    bm.release(p)
    hit, n = bm.match_prefix(t + [9])
    assert n == 4 and list(hit) == p
    bm.release(hit)
    bm.allocate(4)  # forces eviction of the two cached pages
    assert bm.num_cached() == 0


def test_split_balanced():
    lens = [9000, 8000, 7000, 3000, 2000, 1000, 500, 500]
    parts = split_balanced(lens, 16384)
    assert sorted(i for p in parts for i in p) == list(range(len(lens)))
    assert all(sum(lens[i] for i in p) <= 16384 for p in parts)
    parts = split_balanced(lens, 16384, min_count=4)
    assert len(parts) >= 4


def test_shm_segment_roundtrip():
    from axrl_b200.rollout.kv import runtime_module

    rt = runtime_module()
    seg = rt.ShmSegment("/axrl_test_seg", 4096, True)
    try:
        v = np.frombuffer(seg.view(), dtype=np.float32)
        v[:4] = [1, 2, 3, 4]
        seg2 = rt.ShmSegment("/axrl_test_seg", 0, False)
        assert np.frombuffer(seg2.view(), dtype=np.float32)[:4].tolist() == [1, 2, 3, 4]
        seg2.close()
    finally:
        seg.close()
        seg.unlink()


def test_tiny_grpo_cpu_plumbing():
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.grpo_step import SyntheticGRPO, SyntheticGRPOConfig

    torch.manual_seed(0)
    wc = MegatronWorkerConfig()
    wc.lr_scheduler.lr_warmup_steps = 0
    wc.lr_scheduler.max_lr = 1e-3
    g = GrpoTrainerConfig(loss_type="grpo", mismatch_token_clip_max=2.0)
    sc = SyntheticGRPOConfig(num_prompts=8, prompt_len=32, group_size=4, max_new_tokens=64, separate_rollout_copy=True)
    pipe = SyntheticGRPO(resolve_preset("tiny"), wc, g, sc, "cpu")
    before = [p.detach().clone() for p in pipe.rollout.model.parameters()]
    m = pipe.run_step()
    assert m["sequences"] == 32 and m["num_samples"] == 8  # each group prefix-tree merged into one sample
    assert m["grad_norm"] > 0 and np.isfinite(m["loss"])
    # rollout logprobs == trainer old logprobs (same fp32 weights, same math) -> ratio 1
    assert abs(m["ratio_mean"] - 1.0) < 1e-4
    # weight sync reached the rollout copy
    after = list(pipe.rollout.model.parameters())
    assert any(not torch.equal(a, b) for a, b in zip(before, after))
    assert all(torch.equal(a, b) for a, b in zip(after, pipe.train.model.parameters()))


def test_filtered_sampling_controls():
    from axrl_b200.ops.paged import sample_filtered

    torch.manual_seed(0)
    B, V = 4, 64
    logits = torch.randn(B, V)
    logits[:, 5] = 10.0
    ones = torch.ones(B)
    g = torch.Generator().manual_seed(1)
    # top_k = 1 behaves greedily
    tok, lp = sample_filtered(logits, ones, torch.ones(B, dtype=torch.int64), ones, torch.zeros(B), generator=g)
    assert (tok == 5).all()
    assert torch.allclose(lp, torch.log_softmax(logits, -1)[:, 5], atol=1e-5)
    # a huge presence penalty on token 5 (already generated) removes it from a top-1 draw
    hist = torch.full((B, 3), -1, dtype=torch.int64)
    hist[:, 0] = 5
    tok2, _ = sample_filtered(logits, ones, torch.ones(B, dtype=torch.int64), ones, torch.zeros(B), presence=torch.full((B,), 100.0),
                              history=hist, generator=g)
    assert (tok2 != 5).all()
    # allowed-token mask (constrained decoding): only tokens 10..12 may be drawn
    bias = torch.full((B, V), float("-inf"))
    bias[:, 10:13] = 0.0
    for _ in range(5):
        t3, _ = sample_filtered(logits, ones, torch.full((B,), -1), ones, torch.zeros(B), bias=bias, generator=g)
        assert ((t3 >= 10) & (t3 < 13)).all()
    # top-p 0: only the best token; min-p 1.0: only the best token
    t4, _ = sample_filtered(logits, ones, torch.full((B,), -1), torch.zeros(B), torch.zeros(B), generator=g)
    t5, _ = sample_filtered(logits, ones, torch.full((B,), -1), ones, torch.ones(B), generator=g)
    assert (t4 == 5).all() and (t5 == 5).all()


def test_engine_constrained_and_penalised_requests():
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16)
    m = Qwen3Model(cfg)
    m.init_weights(0)
    eng = RolloutEngine(m, max_batch=4, kv_tokens=1024, max_context=128, seed=0, use_cuda_graph=False, burst=4)
    reqs = [GenRequest(rid="allowed", prompt=list(range(3, 15)), max_new_tokens=12, allowed_token_ids=[40, 41, 42]),
            GenRequest(rid="norepeat", prompt=list(range(3, 15)), max_new_tokens=20, top_k=1, presence_penalty=1e4),
            GenRequest(rid="plain", prompt=list(range(5, 9)), max_new_tokens=6)]
    res = {r.rid: r for r in eng.generate(reqs)}
    assert set(res["allowed"].output_ids) <= {40, 41, 42} and len(res["allowed"].output_ids) == 12
    out = res["norepeat"].output_ids
    assert len(out) == 20 and len(set(out)) == 20  # greedy with a huge presence penalty never repeats
    assert len(res["plain"].output_ids) == 6


def test_partial_rollout_carries_unfinished_groups_across_steps():
    """Streaming rollout: each step trains exactly the first `num_prompts` groups to complete; the
    rest keep their partial responses, resume after the weight update, and finish with exactly the
    forced length (so trajectories that spanned several rollout phases are stitched correctly)."""
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.grpo_step import SyntheticGRPO, SyntheticGRPOConfig

    torch.manual_seed(0)
    wc = MegatronWorkerConfig()
    wc.lr_scheduler.lr_warmup_steps = 0
    g = GrpoTrainerConfig(loss_type="grpo", mismatch_token_clip_max=2.0)
    sc = SyntheticGRPOConfig(num_prompts=2, prompt_len=16, group_size=4, forced_len_median=12, forced_len_sigma=1.2,
                             forced_len_min=2, forced_len_max=80, partial_rollout=True, inflight_prompts=5, seed=3,
                             separate_rollout_copy=True, use_cuda_graph=False)
    pipe = SyntheticGRPO(resolve_preset("tiny"), wc, g, sc, "cpu")
    seen_multi = 0
    for _ in range(4):
        m = pipe.run_step()
        assert m["groups_done"] == 2 and m["sequences"] == 8
        assert m["carried_groups"] == 3
        seen_multi += m["multi_segment_trajectories"]
        assert np.isfinite(m["loss"])
    assert seen_multi > 0, "no trajectory spanned two rollout phases"
    # every trajectory still in flight holds a consistent partial state
    for grp in pipe.pool:
        for t in grp.members:
            assert len(t.out_ids) == len(t.out_lps) <= t.req.forced_len
            assert t.done == (len(t.out_ids) == t.req.forced_len)


def test_agentic_multi_turn_step_cpu():
    """Multi-turn tool trajectories in groups sharing a prefix: every step trains the first group to
    finish, packed into prefix trees with the loss on model tokens only; unfinished groups keep
    their turns for the next step."""
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.agentic_step import AgenticConfig, SyntheticAgentic

    torch.manual_seed(0)
    wc = MegatronWorkerConfig()
    wc.lr_scheduler.lr_warmup_steps = 0
    ac = AgenticConfig(group_size=3, inflight_groups=2, prefix_len=16, min_turns=2, max_turns=4, action_min=2, action_max=6, obs_min=2,
                       obs_max=5, max_context=120, pack_len=96, seed=1)
    pipe = SyntheticAgentic(resolve_preset("tiny"), wc, GrpoTrainerConfig(loss_type="grpo"), ac, "cpu")
    for _ in range(3):
        m = pipe.run_step()
        assert m["trajectories"] == 3 and m["carried_groups"] == 1
        assert 2 * 3 <= m["turns"] <= 4 * 3
        assert np.isfinite(m["loss"]) and m["trained_tokens"] > 0
        # the shared prefix and earlier turns are packed once: fewer tokens than the per-turn paths
        assert m["trained_tokens"] < m["turns"] * ac.prefix_len + m["trajectory_tokens"] * 4
    grp = pipe.pool[0]
    assert all(len(t.trace.turn_samples) >= 0 for t in grp)


def test_agentic_group_packing_shares_prefix():
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import resolve_preset
    from axrl_b200.pipeline.agentic_step import AgenticConfig, SyntheticAgentic

    ac = AgenticConfig(group_size=4, inflight_groups=1, prefix_len=20, min_turns=2, max_turns=2, action_min=3, action_max=3, obs_min=2,
                       obs_max=2, max_context=200, pack_len=4096, seed=2)
    pipe = SyntheticAgentic(resolve_preset("tiny"), MegatronWorkerConfig(), GrpoTrainerConfig(), ac, "cpu")
    pipe.pool.append(pipe._new_group())
    while not all(t.done for t in pipe.pool[0]):
        pipe._round([t for t in pipe.pool[0] if not t.done])
    samples = pipe.pack_group(pipe.pool[0])
    assert len(samples) == 1  # one tree for the whole group
    s = samples[0]
    # every generated token trains exactly once; the 20-token prefix is packed once, not per path
    assert int(s.loss_mask.sum()) == 4 * 2 * 3
    real = s.merge_info.real_total
    paths = sum(len(t.turn_samples[i].input_ids) for t in (x.trace for x in pipe.pool[0]) for i in range(2))
    assert real < paths and real <= 20 + 4 * (3 + 2 + 3 + 2)  # prefix once; each trajectory's turns + fork tokens


def _dp_partial_worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
        from axrl_b200.models.qwen3 import resolve_preset
        from axrl_b200.pipeline.grpo_step import SyntheticGRPO, SyntheticGRPOConfig
        from axrl_b200.train.engine import ParallelCtx, TrainEngine

        torch.manual_seed(0)
        wc = MegatronWorkerConfig()
        wc.lr_scheduler.lr_warmup_steps = 0
        par = ParallelCtx(dp_group=dist.group.WORLD, dp_size=world, dp_rank=rank, zero_backend="off")
        train = TrainEngine(wc, resolve_preset("tiny"), "cpu", par=par)
        # rank 1's responses are much longer: its groups finish later
        sc = SyntheticGRPOConfig(num_prompts=2, prompt_len=16, group_size=4, forced_len_median=8 + 40 * rank, forced_len_sigma=0.3,
                                 forced_len_min=2, forced_len_max=80, partial_rollout=True, inflight_prompts=4, seed=3 + rank,
                                 separate_rollout_copy=True, use_cuda_graph=False)
        pipe = SyntheticGRPO(resolve_preset("tiny"), wc, GrpoTrainerConfig(loss_type="grpo"), sc, "cpu", train_engine=train)
        got = []
        for _ in range(3):
            m = pipe.run_step()
            got.append(m["groups_done"])
            assert np.isfinite(m["loss"]) and m["groups_done"] >= 1
        tot = torch.tensor(got)
        dist.all_reduce(tot)
        assert all(int(x) >= sc.num_prompts * world for x in tot), tot  # the global batch every step
        q.put((rank, "ok", got))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))
    finally:
        dist.destroy_process_group()


def test_partial_rollout_data_parallel_global_stop():
    """Data-parallel partial rollout stops on the global batch: the ranks' completed groups add up
    to num_prompts per rank every step, the rank with the shorter responses contributing more."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_partial_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs])
    for p in procs:
        p.join(timeout=60)
    for r, msg, _ in res:
        assert msg == "ok", f"rank {r}:\n{msg}"
    assert sum(res[0][2]) >= sum(res[1][2])  # the faster rank trained at least as many groups

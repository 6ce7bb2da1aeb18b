"""Host runtime (native block manager vs Python twin), micro-batch balancing, and the
tiny CPU GRPO plumbing run (2 layers, hidden 256, 4 heads, FFN 768, vocab 1024, fp32)."""

import numpy as np
import pytest
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

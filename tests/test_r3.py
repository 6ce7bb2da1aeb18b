"""R3: tensor store semantics, routing rows through the trie source map, and exact replay in the MoE
router (a replayed forward reproduces the rollout's expert choices even after the router changed)."""

import numpy as np
import torch

from axrl_b200.data.prefix_tree import merge_trajectory_samples
from axrl_b200.data.sample import Sample
from axrl_b200.models.moe import MoEContext, route
from axrl_b200.train.routing import materialise_row
from axrl_b200.utils.tensor_store import TensorStore


def test_store_local_and_shm():
    for backend in ("local", "shm"):
        st = TensorStore(backend)
        h = st.put(np.arange(20, dtype=np.int16).reshape(10, 2))
        a, b = st.get_batch([h.slice(2, 3), h])
        assert a.tolist() == [[4, 5], [6, 7], [8, 9]] and b.shape == (10, 2)
        st.delete_batch([h])
        assert len(st) == 0


def test_routing_rows_through_trie():
    st = TensorStore()
    p0 = [1, 2, 3, 4, 5]
    p1 = [1, 2, 3, 4, 5, 6, 7, 8]
    lm0 = np.zeros(5, bool)
    lm0[2:4] = True
    lm1 = np.zeros(8, bool)
    lm1[5:7] = True
    s0 = Sample(np.array(p0), np.array(p0[1:] + [-100]), lm0, np.ones(5, bool), np.arange(5), 0, 0, lm0.astype(np.float32))
    s1 = Sample(np.array(p1), np.array(p1[1:] + [-100]), lm1, np.ones(8, bool), np.arange(8), 0, 0, lm1.astype(np.float32))
    r0 = np.stack([np.full((2, 1), 10 + i) for i in range(4)])  # 4 rows for 5 tokens
    r1 = np.stack([np.full((2, 1), 20 + i) for i in range(7)])
    s0.routing_handles_per_path = [[st.put(r0)]]
    s1.routing_handles_per_path = [[st.put(r1)]]
    m = merge_trajectory_samples([s0, s1], align_size=1)
    rows, valid = materialise_row(st, m.routing_handles_per_path, m.merge_info, len(m.input_ids))
    assert valid[: m.merge_info.real_total - 1].all() and not valid[m.merge_info.real_total - 1]
    # position p's routing row = source path's row p (token p processed on that path)
    for p in range(m.merge_info.real_total - 1):
        src = m.merge_info.routing_source_path[p]
        assert rows[p, 0, 0] == (10 if src == 0 else 20) + m.merge_info.routing_source_read_pos[p] - 1


def test_router_replay_exact():
    torch.manual_seed(0)
    logits = torch.randn(6, 8)
    _, ids = route(logits, 2, True)
    new_logits = logits + torch.randn(6, 8)  # router drifted after an update
    _, live = route(new_logits, 2, True)
    w, rep = route(new_logits, 2, True, replay=ids)
    assert torch.equal(rep, ids) and not torch.equal(live, ids)
    mask = torch.tensor([True, False, True, False, True, False])
    _, mixed = route(new_logits, 2, True, replay=ids, replay_mask=mask)
    assert torch.equal(mixed[mask], ids[mask]) and torch.equal(mixed[~mask], live[~mask])
    assert torch.allclose(w.sum(-1), torch.ones(6))


def test_moe_forward_replay_capture_roundtrip():
    from axrl_b200.models.qwen3 import Qwen3Model, resolve_preset
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

    m = Qwen3Model(resolve_preset("tiny-moe"))
    m.init_weights(0)
    ids = torch.randint(0, 1024, (12,))
    pos = torch.arange(12)
    spec = causal_spec_from_cu_seqlens([0, 12])
    cap = MoEContext(capture={})
    with torch.no_grad():
        h1 = m(ids, pos, spec, cap)
        for layer in m.layers:
            layer.mlp.router.add_(torch.randn_like(layer.mlp.router))  # routing would change...
        rep = MoEContext(replay={k: v.long() for k, v in cap.capture.items()}, capture={})
        m(ids, pos, spec, rep)
    for k in cap.capture:  # ...but replay reproduces the captured experts
        assert torch.equal(rep.capture[k], cap.capture[k])
    assert h1.shape == (12, 256)

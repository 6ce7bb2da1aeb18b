"""Label-aware prefix-tree packing of multi-turn trajectories.

A trajectory produces one training path per assistant turn; later turns
repeat the earlier context.  Packing the paths into a trie computes every
shared prefix once.  Behaviour matches reference
``axrl/utils/megatron/prefix_tree.py:20-831`` (the attention ranges, the
position ids and the routing source map must agree exactly, because they
decide which tokens attend to which and which label each position trains on):

* **label-aware sharing** – two paths share packed position ``p`` only if one
  of them ends at ``p`` or both continue with the same next token (the label of
  ``p``).  At a fork the last common token is therefore duplicated;
* packed layout is DFS pre-order, each node a contiguous span; the last node
  absorbs the alignment padding (``lcm(align, 128)``);
* attention per node: **full** to each ancestor span (type 0, nearest
  ancestor first) then **causal** to itself (type 1);
* RoPE position of a packed token = its offset inside its own path;
* trainable-wins scatter: at most one path may be trainable on a shared slot;
  the routing row of a packed position comes from the trainable path, else
  from the lowest-index path that visits it.

The implementation here keeps token runs as numpy arrays (vectorised common
prefix) and uses one generic "walk" routine for both insertion and the
non-mutating size estimate used by greedy packing.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Iterator, Sequence

import numpy as np
import torch

from axrl_b200.configs import IGNORE_INDEX


@dataclass
class PrefixTreeNode:
    start: int
    end: int
    parent: int


@dataclass
class PrefixMergeInfo:
    """Packed-layout metadata of one merged trajectory (or a forest of them)."""

    nodes: list[PrefixTreeNode]
    path_to_leaf: list[tuple[int, int]]
    q_ranges: list[tuple[int, int]]
    k_ranges: list[tuple[int, int]]
    attn_type_map: list[int]
    total_padded: int
    max_path_len: int
    turn_sample_lens: list[int]
    real_total: int = 0
    routing_source_path: np.ndarray | None = None
    routing_source_read_pos: np.ndarray | None = None


class _Node:
    __slots__ = ("toks", "kids", "owners")

    def __init__(self, toks: np.ndarray) -> None:
        self.toks = toks
        self.kids: list[_Node] = []
        self.owners: list[int] = []


def _shared_len(a: np.ndarray, b: np.ndarray) -> int:
    """Longest common prefix, shortened by one when both runs continue past it
    (the last shared token would otherwise need two different labels)."""
    n = min(len(a), len(b))
    if n == 0:
        return 0
    neq = np.flatnonzero(a[:n] != b[:n])
    k = int(neq[0]) if neq.size else n
    if 0 < k < len(a) and k < len(b):
        k -= 1
    return k


def _find_child(kids: Sequence[_Node], suffix: np.ndarray) -> tuple[_Node | None, int]:
    first = suffix[0]
    for c in kids:
        if len(c.toks) and c.toks[0] == first:
            k = _shared_len(c.toks, suffix)
            if k > 0:
                return c, k
    return None, 0


class MergingTree:
    """Incremental label-aware trie; ``packed_len`` is the unpadded packed size."""

    def __init__(self) -> None:
        self.root = _Node(np.zeros(0, dtype=np.int64))
        self.packed_len = 0
        self.path_count = 0

    def add_path(self, path: Sequence[int]) -> None:
        suffix = np.asarray(path, dtype=np.int64)
        node = self.root
        while len(suffix):
            child, k = _find_child(node.kids, suffix)
            if child is None:
                leaf = _Node(suffix.copy())
                leaf.owners.append(self.path_count)
                node.kids.append(leaf)
                self.packed_len += len(suffix)
                self.path_count += 1
                return
            if k < len(child.toks):  # split the child at k
                tail = _Node(child.toks[k:])
                tail.kids, tail.owners = child.kids, child.owners
                child.toks, child.kids, child.owners = child.toks[:k], [tail], []
            node, suffix = child, suffix[k:]
        node.owners.append(self.path_count)
        self.path_count += 1

    def get_packed_len_if_add_path(self, path: Sequence[int]) -> int:
        """Packed length after a hypothetical :meth:`add_path` (tree unchanged)."""
        suffix = np.asarray(path, dtype=np.int64)
        # Walk state: a list of candidate (tokens, children) runs at the current depth.
        cands: list[tuple[np.ndarray, list[_Node]]] = [(c.toks, c.kids) for c in self.root.kids]
        while len(suffix):
            hit = None
            for toks, kids in cands:
                if len(toks) and toks[0] == suffix[0]:
                    k = _shared_len(toks, suffix)
                    if k > 0:
                        hit = (toks, kids, k)
                        break
            if hit is None:
                return self.packed_len + len(suffix)
            toks, kids, k = hit
            cands = [(toks[k:], kids)] if k < len(toks) else [(c.toks, c.kids) for c in kids]
            suffix = suffix[k:]
        return self.packed_len

    def to_packed_sequence(self) -> tuple[list[int], list[PrefixTreeNode], list[tuple[int, int]]]:
        packed: list[np.ndarray] = []
        nodes: list[PrefixTreeNode] = []
        p2l: list[tuple[int, int]] = [(-1, 0)] * self.path_count
        cursor = 0
        stack: list[tuple[_Node, int, int]] = [(c, -1, 0) for c in reversed(self.root.kids)]
        while stack:
            nd, parent, prefix = stack.pop()
            idx = len(nodes)
            nodes.append(PrefixTreeNode(cursor, cursor + len(nd.toks), parent))
            packed.append(nd.toks)
            cursor += len(nd.toks)
            for o in nd.owners:
                p2l[o] = (idx, prefix)
            stack.extend((c, idx, prefix + len(nd.toks)) for c in reversed(nd.kids))
        flat = np.concatenate(packed).tolist() if packed else []
        return flat, nodes, p2l


def build_tree_packed_sequence(paths: Sequence[Sequence[int]]) -> tuple[list[int], list[PrefixTreeNode], list[tuple[int, int]]]:
    tree = MergingTree()
    for p in paths:
        tree.add_path(p)
    return tree.to_packed_sequence()


def get_packed_len_if_merge(tree: MergingTree, sample: Any) -> int:
    return tree.get_packed_len_if_add_path(np.asarray(sample.input_ids))


def add_sample_to_merging_tree(tree: MergingTree, sample: Any) -> None:
    tree.add_path(np.asarray(sample.input_ids))


def pack_tree_aligned_as_list(paths, align_size: int, pad_token_id: int = 0, trie=None):  # noqa: ANN001
    packed, nodes, p2l = trie if trie is not None else build_tree_packed_sequence(paths)
    total = len(packed)
    pad = (-total) % math.lcm(align_size, 128)
    if pad and nodes:
        last = nodes[-1]
        nodes[-1] = PrefixTreeNode(last.start, last.end + pad, last.parent)
        packed = list(packed) + [pad_token_id] * pad
    return packed, nodes, p2l, total + pad


def _ancestors(nodes: Sequence[PrefixTreeNode], i: int) -> list[int]:
    out, p = [], nodes[i].parent
    while p >= 0:
        out.append(p)
        p = nodes[p].parent
    return out


def build_prefix_tree_ranges_as_lists(nodes: Sequence[PrefixTreeNode]):  # noqa: ANN201
    q, k, t = [], [], []
    for i, nd in enumerate(nodes):
        for a in _ancestors(nodes, i):
            an = nodes[a]
            if an.end > an.start:
                q.append((nd.start, nd.end))
                k.append((an.start, an.end))
                t.append(0)
        q.append((nd.start, nd.end))
        k.append((nd.start, nd.end))
        t.append(1)
    return q, k, t


def build_prefix_tree_ranges(nodes: Sequence[PrefixTreeNode], device: Any = "cpu"):  # noqa: ANN201
    q, k, t = build_prefix_tree_ranges_as_lists(nodes)
    return (torch.tensor(q, dtype=torch.int32, device=device).reshape(-1, 2),
            torch.tensor(k, dtype=torch.int32, device=device).reshape(-1, 2),
            torch.tensor(t, dtype=torch.int32, device=device))


def _prefix_len(nodes: Sequence[PrefixTreeNode], i: int) -> int:
    return sum(nodes[a].end - nodes[a].start for a in _ancestors(nodes, i))


def compute_tree_rel_positions_as_list(nodes: Sequence[PrefixTreeNode], total: int) -> list[int]:
    pos = np.zeros(total, dtype=np.int64)
    for i, nd in enumerate(nodes):
        pos[nd.start:nd.end] = _prefix_len(nodes, i) + np.arange(nd.end - nd.start)
    return pos.tolist()


def compute_tree_rel_positions(nodes, total: int, device: Any = "cpu") -> torch.Tensor:  # noqa: ANN001
    return torch.tensor(compute_tree_rel_positions_as_list(nodes, total), dtype=torch.int32, device=device)


def path_chain_root_to_leaf(nodes: Sequence[PrefixTreeNode], leaf: int) -> list[int]:
    chain = [leaf] + _ancestors(nodes, leaf)
    chain.reverse()
    return chain


def compute_max_path_length(nodes, path_to_leaf) -> int:  # noqa: ANN001
    best = 0
    for leaf, _ in path_to_leaf:
        best = max(best, sum(nodes[n].end - nodes[n].start for n in path_chain_root_to_leaf(nodes, leaf)))
    return best


def iter_path_segments_in_packed(nodes, path_to_leaf, path_lens) -> Iterator[tuple[int, int, int, int]]:  # noqa: ANN001
    """Yield ``(path, write_start, read_start, take)`` over every path's root->leaf chain."""
    for pi, (leaf, _) in enumerate(path_to_leaf):
        read = 0
        for n in path_chain_root_to_leaf(nodes, leaf):
            take = min(nodes[n].end - nodes[n].start, path_lens[pi] - read)
            if take <= 0:
                break
            yield pi, nodes[n].start, read, take
            read += take


def scatter_packed_to_batch(packed: torch.Tensor, nodes, path_to_leaf, attention_mask: torch.Tensor) -> torch.Tensor:  # noqa: ANN001
    B, S = attention_mask.shape[:2]
    out = torch.zeros((B, S, *packed.shape[1:]), dtype=packed.dtype, device=packed.device)
    valid = [attention_mask[i].nonzero().flatten() for i in range(B)]
    for pi, w, r, take in iter_path_segments_in_packed(nodes, path_to_leaf, [int(v.numel()) for v in valid]):
        out[pi, valid[pi][r:r + take]] = packed[w:w + take]
    return out


def build_prefix_merge_info(*, nodes, path_to_leaf, total_padded, turn_sample_lens, real_total) -> PrefixMergeInfo:  # noqa: ANN001
    q, k, t = build_prefix_tree_ranges_as_lists(nodes)
    assert len(turn_sample_lens) == len(path_to_leaf)
    return PrefixMergeInfo(list(nodes), list(path_to_leaf), q, k, t, total_padded,
                           compute_max_path_length(nodes, path_to_leaf), list(turn_sample_lens), real_total)


def merge_prefix_merge_infos(infos: Sequence[PrefixMergeInfo]) -> PrefixMergeInfo:
    """Concatenate per-trajectory infos into one forest with shifted offsets."""
    nodes, p2l, q, k, t, lens = [], [], [], [], [], []
    pos = node_off = 0
    for inf in infos:
        nodes += [PrefixTreeNode(n.start + pos, n.end + pos, n.parent + node_off if n.parent >= 0 else -1) for n in inf.nodes]
        p2l += [(leaf + node_off, pl) for leaf, pl in inf.path_to_leaf]
        q += [(a + pos, b + pos) for a, b in inf.q_ranges]
        k += [(a + pos, b + pos) for a, b in inf.k_ranges]
        t += list(inf.attn_type_map)
        lens += list(inf.turn_sample_lens)
        pos += inf.total_padded
        node_off += len(inf.nodes)
    return PrefixMergeInfo(nodes, p2l, q, k, t, pos, max((i.max_path_len for i in infos), default=0), lens,
                           sum(i.real_total for i in infos))


_OPT_F32 = ("rollout_logprobs", "teacher_logprobs", "old_values", "returns", "turn_reward")


def merge_trajectory_samples(per_turn_samples: Sequence[Any], align_size: int = 128):  # noqa: ANN201
    """Trie-pack one trajectory's per-turn samples into one merged ``Sample``."""
    from axrl_b200.data.sample import Sample

    assert per_turn_samples, "need at least one sample"
    paths = [np.asarray(s.input_ids) for s in per_turn_samples]
    packed, nodes, p2l, total = pack_tree_aligned_as_list(paths, align_size)
    lens = [len(p) for p in paths]

    labels = np.full(total, IGNORE_INDEX, dtype=np.int32)
    loss_mask = np.zeros(total, dtype=bool)
    attn = np.zeros(total, dtype=bool)
    adv = np.zeros(total, dtype=np.float32)
    opt = {n: np.zeros(total, dtype=np.float32) for n in _OPT_F32 if all(getattr(s, n) is not None for s in per_turn_samples)}
    turn_index = np.full(total, -1, dtype=np.int32) if all(s.turn_index is not None for s in per_turn_samples) else None
    src_path = np.full(max(total - 1, 0), -1, dtype=np.int64)
    src_read = np.full(max(total - 1, 0), -1, dtype=np.int64)

    for pi, w, r, take in iter_path_segments_in_packed(nodes, p2l, lens):
        s = per_turn_samples[pi]
        ws = np.arange(w, w + take)
        rs = np.arange(r, r + take)
        attn[ws] = True
        tr = s.loss_mask[rs]
        if tr.any():
            tw, trd = ws[tr], rs[tr]
            if loss_mask[tw].any():
                bad = int(tw[loss_mask[tw]][0])
                raise AssertionError(f"shared trainable slot at packed pos {bad}: at most one path may be trainable there")
            labels[tw] = s.labels[trd]
            loss_mask[tw] = True
            adv[tw] = s.advantage[trd]
            for n, buf in opt.items():
                buf[tw] = getattr(s, n)[trd]
            if turn_index is not None:
                turn_index[tw] = s.turn_index[trd]
            pos = tw > 0
            src_path[tw[pos] - 1] = pi
            src_read[tw[pos] - 1] = trd[pos]
        # Non-trainable visitors fill only unclaimed routing slots (first visitor wins).
        nt_w, nt_r = ws[~tr], rs[~tr]
        keep = nt_w > 0
        nt_w, nt_r = nt_w[keep], nt_r[keep]
        free = src_path[nt_w - 1] == -1
        src_path[nt_w[free] - 1] = pi
        src_read[nt_w[free] - 1] = nt_r[free]
        # Untrainable labels are IGNORE; keep labels of shared context for debugging parity.

    real_total = int(attn.sum())
    info = build_prefix_merge_info(nodes=nodes, path_to_leaf=p2l, total_padded=total, turn_sample_lens=lens, real_total=real_total)
    if real_total > 1:
        info.routing_source_path = src_path[: real_total - 1].copy()
        info.routing_source_read_pos = src_read[: real_total - 1].copy()
    handles = None
    if any(s.routing_handles_per_path is not None for s in per_turn_samples):
        handles = []
        for s in per_turn_samples:
            assert s.routing_handles_per_path is not None and len(s.routing_handles_per_path) == 1
            handles.append(list(s.routing_handles_per_path[0]))
    return Sample(
        input_ids=np.asarray(packed, dtype=np.int32), labels=labels, loss_mask=loss_mask, attention_mask=attn,
        position_ids=np.asarray(compute_tree_rel_positions_as_list(nodes, total), dtype=np.int32),
        reward=0.0, reward_baseline=0.0, advantage=adv,
        turn_index=turn_index, routing_handles_per_path=handles, merge_info=info, **opt,
    )


def unpack_tensor_from_merged(packed: torch.Tensor, info: PrefixMergeInfo) -> list[list[float]]:
    """Per-turn views of a per-token quantity stored in packed layout."""
    if packed.dim() == 2 and packed.size(0) == 1:
        packed = packed[0]
    assert packed.dim() == 1
    out = []
    for pi, (leaf, _) in enumerate(info.path_to_leaf):
        n = info.turn_sample_lens[pi]
        vals: list[float] = []
        for node in path_chain_root_to_leaf(info.nodes, leaf):
            nd = info.nodes[node]
            take = min(nd.end - nd.start, n - len(vals))
            if take <= 0:
                break
            vals += packed[nd.start:nd.start + take].tolist()
        out.append(vals + [0.0] * (n - len(vals)))
    return out


def gather_merged_routing_per_path(per_path_routings: Sequence[np.ndarray], info: PrefixMergeInfo) -> np.ndarray:
    """Merged routing rows from per-path concatenated routing arrays via the source map.
    Row for merged position ``p+1`` is ``per_path[src_path[p]][src_read[p] - 1]``."""
    assert info.routing_source_path is not None and info.routing_source_read_pos is not None
    r0 = per_path_routings[0]
    if info.real_total <= 1:
        return np.empty((0, *r0.shape[1:]), dtype=r0.dtype)
    sp, sr = info.routing_source_path, info.routing_source_read_pos
    assert (sp >= 0).all(), "every merged routing row needs a source"
    out = np.empty((sp.shape[0], *r0.shape[1:]), dtype=r0.dtype)
    for p in np.unique(sp):
        m = sp == p
        out[m] = per_path_routings[int(p)][sr[m] - 1]
    return out


def extract_merge_info_from_batch(batch: Any) -> list[PrefixMergeInfo] | None:
    infos = batch.objects.get("merge_info") if hasattr(batch, "objects") else None
    if infos is None or all(i is None for i in infos):
        return None
    return list(infos)


def extract_paths_from_batch(input_ids: torch.Tensor, attention_mask: torch.Tensor) -> list[list[int]]:
    return [input_ids[i][attention_mask[i]].tolist() for i in range(input_ids.size(0))]

"""Per-layer hidden-state diff between the flat (one row per path) and the prefix-tree merged
forward of the same trajectories.

Reference: ``magi_prefix_merging_layer_diff`` (``axrl/utils/megatron/layer_diff.py:46-180``),
which compares TE / flat-Magi / merged-Magi forwards through forward hooks.  Here both forwards
run the same model over this package's range-list attention: the flat forward packs every path
as its own causal sequence; the merged forward packs the trie (shared prefixes once).  Forward
hooks collect each decoder layer's output; merged positions are mapped back to every path with
the trie's node chain, so each path's tokens are compared at every layer.  With exact arithmetic
the two are identical; the report shows where numerical differences enter and how they grow.
"""

from __future__ import annotations

from typing import Any

import torch

from axrl_b200.data.prefix_tree import path_chain_root_to_leaf


def _collect(model: torch.nn.Module, run) -> list[torch.Tensor]:  # noqa: ANN001
    outs: list[torch.Tensor] = []
    hooks = [layer.register_forward_hook(lambda m, i, o: outs.append(o.detach().float())) for layer in model.layers]
    try:
        with torch.no_grad():
            final = run()
        outs.append(final.detach().float())
    finally:
        for h in hooks:
            h.remove()
    return outs


def merged_index_for_paths(info: Any) -> list[torch.Tensor]:
    """For every path: the merged-layout position of each of its tokens."""
    out = []
    for pi, (leaf, _) in enumerate(info.path_to_leaf):
        n = info.turn_sample_lens[pi]
        idx: list[int] = []
        for node in path_chain_root_to_leaf(info.nodes, leaf):
            nd = info.nodes[node]
            take = min(nd.end - nd.start, n - len(idx))
            if take <= 0:
                break
            idx.extend(range(nd.start, nd.start + take))
        out.append(torch.tensor(idx, dtype=torch.long))
    return out


def prefix_merging_layer_diff(model: torch.nn.Module, paths: list[list[int]], merged_sample: Any) -> list[dict[str, float]]:
    """Per layer (and the final norm): max / mean |h_flat - h_merged| over all path tokens."""
    from axrl_b200.ops.attention_spec import spec_from_triples

    dev = next(model.parameters()).device
    # flat: every path its own causal segment
    ids, pos, triples, offs, off = [], [], [], [], 0
    for p in paths:
        ids += p
        pos += list(range(len(p)))
        triples.append((off, off + len(p), off, off + len(p), 1))
        offs.append(off)
        off += len(p)
    flat_spec = spec_from_triples(triples, off)
    if dev.type == "cuda":
        flat_spec = flat_spec.to(dev)
    t_ids = torch.tensor(ids, device=dev)
    t_pos = torch.tensor(pos, dtype=torch.int32, device=dev)
    flat = _collect(model, lambda: model(t_ids, t_pos, flat_spec))
    # merged: the trie layout of the sample
    info = merged_sample.merge_info
    m_spec = spec_from_triples([(q0, q1, k0, k1, int(t)) for (q0, q1), (k0, k1), t in zip(info.q_ranges, info.k_ranges, info.attn_type_map)],
                               info.total_padded)
    if dev.type == "cuda":
        m_spec = m_spec.to(dev)
    m_ids = torch.as_tensor(merged_sample.input_ids, device=dev).long()
    m_pos = torch.as_tensor(merged_sample.position_ids, device=dev).int()
    merged = _collect(model, lambda: model(m_ids, m_pos, m_spec))
    where = merged_index_for_paths(info)
    rows = []
    for li, (a, b) in enumerate(zip(flat, merged)):
        diffs = []
        for pi, p in enumerate(paths):
            fa = a[offs[pi]:offs[pi] + len(p)]
            mb = b[where[pi].to(b.device)]
            diffs.append((fa - mb).abs())
        d = torch.cat(diffs, 0)
        rows.append({"layer": li if li < len(flat) - 1 else "final_norm", "max_abs": float(d.max()), "mean_abs": float(d.mean()),
                     "ref_mean_abs": float(torch.cat([a[offs[i]:offs[i] + len(p)] for i, p in enumerate(paths)]).abs().mean())})
    return rows

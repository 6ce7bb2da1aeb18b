"""Rollout Routing Replay (R3): turn captured expert ids into per-layer replay targets.

Reference: ``RoutingMaterialiser`` (``axrl/utils/megatron/routing_materialiser.py:45-235``) and
``router_replay.py:67-554``.  For every row of a packed micro-batch the materialiser fetches the
row's routing handles (one chain per path), concatenates them, and for prefix-tree merged rows
gathers the merged layout through the trie's source map.  A path of ``n`` tokens carries ``n - 1``
routing rows: row ``k`` holds the experts chosen when token ``k`` was processed (the step that
predicted token ``k + 1``).  The last token of a path has no recorded routing, so it (and any
unrecorded position) uses the live router; with ``loss_tokens_only`` replay is restricted to
positions whose next token is trained (``replay_routing_for_loss_tokens_only``).

Output: ``MoEContext.replay = {moe_layer_index: (T, K) int64}`` and ``replay_mask (T,)`` for the
packed token stream, copied to the device in one transfer per micro-batch.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from axrl_b200.data.prefix_tree import gather_merged_routing_per_path
from axrl_b200.models.moe import MoEContext


def materialise_row(store: Any, handles_per_path: list[list[Any]], merge_info: Any, row_len: int) -> tuple[np.ndarray, np.ndarray]:
    """(row_len, L, K) routing and (row_len,) validity for one sample row."""
    per_path = []
    for chain in handles_per_path:
        parts = store.get_batch(chain)
        per_path.append(np.concatenate(parts, 0) if parts else None)
    if merge_info is not None:
        rows = gather_merged_routing_per_path(per_path, merge_info)
    else:
        rows = per_path[0]
    L, K = rows.shape[1], rows.shape[2]
    out = np.zeros((row_len, L, K), dtype=np.int64)
    valid = np.zeros(row_len, dtype=bool)
    n = min(rows.shape[0], row_len)
    out[:n] = rows[:n]
    valid[:n] = True
    return out, valid


def build_moe_context(store: Any, mb: Any, handles: list, infos: list, moe_layers: list[int], device: Any,
                      loss_tokens_only: bool = False) -> MoEContext:
    """Replay targets for a :class:`PackedMicroBatch` (``handles``/``infos`` per row)."""
    T = mb.num_tokens
    chunks, valid = [], []
    for li, r in enumerate(mb.rows):
        n = mb.row_len[li]
        if handles[li] is None:
            chunks.append(None)
            valid.append(np.zeros(n, bool))
            continue
        rr, vv = materialise_row(store, handles[li], infos[li], n)
        chunks.append(rr)
        valid.append(vv)
    ref = next((c for c in chunks if c is not None), None)
    if ref is None:
        return MoEContext()
    L, K = ref.shape[1], ref.shape[2]
    allr = np.concatenate([c if c is not None else np.zeros((len(v), L, K), np.int64) for c, v in zip(chunks, valid)], 0)
    mask = np.concatenate(valid)
    if allr.shape[0] < T:  # trailing padding tokens of the packed stream: live router
        allr = np.concatenate([allr, np.zeros((T - allr.shape[0], L, K), np.int64)], 0)
        mask = np.concatenate([mask, np.zeros(T - mask.shape[0], bool)])
    if loss_tokens_only:
        mask &= mb.loss_mask.cpu().numpy().astype(bool)
    assert allr.shape[0] == T
    t = torch.from_numpy(allr)
    if torch.device(device).type == "cuda":
        t = t.pin_memory()
    t = t.to(device, non_blocking=True)
    m = torch.from_numpy(mask).to(device, non_blocking=True)
    assert len(moe_layers) == L, f"routing has {L} layers, model has {len(moe_layers)} MoE layers"
    return MoEContext(replay={layer: t[:, i] for i, layer in enumerate(moe_layers)}, replay_mask=m)

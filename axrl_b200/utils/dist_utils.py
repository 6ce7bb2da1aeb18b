"""Distributed layout helpers: rank coordinates and object collectives.

Reference: ``MCoreDistInfo`` and the object-gather helpers of ``axrl/utils/dist_utils.py:14-175``.
The layout order is TP fastest, then CP, then DP, then PP (Megatron's default): the global rank of
coordinates (tp, cp, dp, pp) is ``tp + TP*(cp + CP*(dp + DP*pp))``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch.distributed as dist


@dataclass(frozen=True)
class DistLayout:
    tp: int = 1
    cp: int = 1
    dp: int = 1
    pp: int = 1

    @property
    def world(self) -> int:
        return self.tp * self.cp * self.dp * self.pp

    def coords(self, rank: int) -> dict[str, int]:
        tp = rank % self.tp
        r = rank // self.tp
        cp = r % self.cp
        r //= self.cp
        dp = r % self.dp
        pp = r // self.dp
        return {"tp": tp, "cp": cp, "dp": dp, "pp": pp}

    def rank_of(self, tp: int = 0, cp: int = 0, dp: int = 0, pp: int = 0) -> int:
        return tp + self.tp * (cp + self.cp * (dp + self.dp * pp))

    def group_ranks(self, axis: str) -> list[list[int]]:
        """Every group of ranks that differ only in ``axis`` (e.g. all TP groups)."""
        sizes = {"tp": self.tp, "cp": self.cp, "dp": self.dp, "pp": self.pp}
        others = [a for a in ("tp", "cp", "dp", "pp") if a != axis]
        groups = []
        import itertools

        for vals in itertools.product(*[range(sizes[a]) for a in others]):
            base = dict(zip(others, vals))
            groups.append([self.rank_of(**{**base, axis: i}) for i in range(sizes[axis])])
        return groups

    def new_groups(self) -> dict[str, Any]:
        """Create this rank's TP/CP/DP/PP process groups (every rank must call it)."""
        me = self.coords(dist.get_rank())
        out = {}
        for axis in ("tp", "cp", "dp", "pp"):
            for ranks in self.group_ranks(axis):
                g = dist.new_group(ranks)
                if dist.get_rank() in ranks:
                    out[axis] = g
        out["coords"] = me
        return out


def all_gather_objects(obj: Any, group: Any = None) -> list[Any]:
    if not dist.is_initialized():
        return [obj]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def broadcast_object(obj: Any, src: int = 0, group: Any = None) -> Any:
    if not dist.is_initialized():
        return obj
    box = [obj]
    dist.broadcast_object_list(box, src=src, group=group)
    return box[0]

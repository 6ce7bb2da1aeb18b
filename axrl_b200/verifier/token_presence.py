"""Synthetic reward used by the plumbing and benchmark configs: 1.0 iff a given token id appears in the response."""

from __future__ import annotations

from typing import Sequence


def token_presence_reward(response_ids: Sequence[int], token_id: int = 7) -> float:
    return 1.0 if token_id in response_ids else 0.0
